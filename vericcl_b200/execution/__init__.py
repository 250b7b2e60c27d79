"""Run infrastructure: context, events, budgets, processes, ownership, checkpoints, publication."""
