"""Python handle on the CPU oracle (oracle/_build/librefcpu.so).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs; the product package never imports
this module.  The library is a C++ restatement of the FerrisBoost reference CPU
engine (see oracle/refcpu.cpp for per-function citations), pinned against the
XGBoost 3.4.1 golden margins in tests/golden/.
"""
from .refcpu import RefCPU, rc_params, build, LIB_PATH  # noqa: F401
