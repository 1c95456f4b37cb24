"""Oracle package: CPU checker for the bee_b200 CUDA kernels.

TEST INFRASTRUCTURE ONLY — imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the bee_b200 product path.
"""
