"""B200 (sm_100a) sparse 3x3x3 submanifold convolution for pwilkin/trellis.cpp's decoders.

The product is libtb_sparse.so (C ABI: include/tb_sparse.h). This package holds its build
script, a ctypes binding (`_lib`), the host-side operator mirror used by tests and the
benchmark (`ops`), multi-GPU z-slab sharding (`dist`) and seeded inputs (`synth`).
"""
from . import build  # noqa: F401
