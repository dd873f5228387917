"""polar_pack_b200 -- B200-native (sm_100a) fused dequant-matmul path for
polar_pack's packed multi-model weight streams.

Drop-in modules mirroring the reference call surface:

* ``polar_pack_b200.quad_kernels``  -- ``pack_quad_layer``, ``quad_bitpacked``
* ``polar_pack_b200.polar_kernels`` -- ``pack_amp_phase``,
  ``quantize_polar_bitpacked``, ``polar_dual_bitpacked``

The compute runs in the in-tree CUDA library ``libpolarpack_b200.so``
(C ABI in ``include/polar_pack_b200.h``); there is no CPU fallback.
"""
__version__ = "0.1.0"
