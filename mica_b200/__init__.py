"""mica_b200: B200 (sm_100a) W8A8 linear-layer hot path of Mica's serving runtime.

Submodules mirror the reference's surface (v0.5/serving/lib/):
  int8_kernels   act_quant / mm_i8 / available / preload / STATS  (lib/int8_kernels.py)
  int8_runtime   QLinear, convert                                (lib/int8_runtime.py)
  fused_kernels  rms_norm, swi_glu                               (lib/fused_kernels.py)
The kernels are in libmica_w8a8.so (csrc/, C ABI in include/mica_w8a8.h).
"""
__version__ = '0.1.0'
