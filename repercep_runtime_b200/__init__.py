"""repercep_runtime_b200 — the FP8 attention hot path of repercep-runtime,
rebuilt for NVIDIA B200 (sm_100a).

Layers (top to bottom):
  attention/, backend/   drop-in mirrors of the reference's AttentionOp and
                         Backend plugin seams (src/repercep/attention,
                         src/repercep/backend) with the new B200 op/backend
  parallel               batch x head sharding and context parallelism
  ops                    torch-facing wrappers + torch custom ops
  _lib                   ctypes binding of librepercep_b200.so (C ABI,
                         include/repercep_b200.h)
  csrc/                  sm_100a CUDA: quantize, tcgen05 attention, C ABI
"""

__version__ = "0.1.0"
