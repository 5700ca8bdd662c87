"""TEST INFRASTRUCTURE ONLY: the CPU oracle (a C++ restatement of the
reference's token-loop arithmetic) and its ctypes access. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use it."""
