"""Online stage: probes, calibration, traces, clock alignment, measured acceptance."""
