"""vericcl_b200: a Blackwell-native collective schedule synthesizer and executor.

The CPU side synthesizes AllGather/AllReduce (and the other MSCCL collectives)
schedules from four JSON documents (topology, sketch, atom, runtime), lowers
them to MSCCL-style XML, verifies them, predicts their completion time with an
exact event model and repairs them against measurements.  The GPU side runs a
compiled form of the XML with one persistent sm_100a interpreter kernel that
moves data with direct peer loads over NVLink 5 / NVSwitch and NVLS multimem
reductions, fusing the reduction, cast and scale into the same traffic.
"""
__version__ = "0.1.0"

__all__ = ["__version__"]
