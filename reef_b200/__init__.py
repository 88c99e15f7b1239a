"""reef_b200: reef's W8A8 / int8 hot path as sm_100a kernels behind a C ABI.

- ``reef_b200/csrc``: CUDA kernels (tcgen05 int8 GEMM, quantiser, attention)
  and the extern "C" surface of include/reef_b200.h, built into
  ``reef_b200/libreef_b200.so`` by ``python -m reef_b200.build``.
- :mod:`reef_b200._lib`: ctypes binding of that ABI.
- :mod:`reef_b200.kernels`: reef_kernels-named entry points over CUDA tensors.
"""
__all__ = ["kernels"]
