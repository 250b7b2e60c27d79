"""Synthesis solvers: MILP layer (HiGHS), demands, route MILP, constructive trees."""
