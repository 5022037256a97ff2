"""nova_b200 -- B200-native (sm_100a) quantized-inference path of pplmx/nova.

The product is the C ABI in include/nova_q.h, implemented by
nova_b200/libnova_q.so (hand-written CUDA for sm_100a), and the drop-in C++
headers under include/cuda/quantize/.  This Python package only loads that
library (nova_b200.capi) for tests and benchmarks.  There is no fallback:
importing nova_b200.capi fails loudly when the library has not been built.
"""
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libnova_q.so")

__all__ = ["LIB_PATH"]
