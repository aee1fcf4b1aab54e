"""The callers of the op: workload generation, runners, timers and the multi-layer decode step.

These mirror the reference's operator harness (benchmarks/workload.py, positions.py, impls.py,
benchmark_utils.py) so the reference's tests and sweeps read the same against this build.
The validation gate, which needs the CPU oracle, lives with the tests.
"""
