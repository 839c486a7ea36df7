"""fast_b200: B200-native temporal-attention hot path of FAST (TGAT/TGN/APAN training).

Layers:
  include/fast_b200.h + libfast_b200.so   C ABI over hand-written sm_100a kernels
  fast_b200._ext.{fastAgg,sampler_core}   drop-in pybind11 modules of the reference API
  fast_b200.ops / model / train           device-resident training path in PyTorch
"""
__version__ = "0.1.0"
