"""walsh_research_b200: B200-native (sm_100a) inference of Walsh's forward hot path.

The public model API lives in ``walsh_research_b200.model`` and mirrors the
reference's ``src.model`` package; kernels are reached through the C ABI in
``include/walsh.h`` (libwalsh.so, loaded by ``walsh_research_b200._lib``).
"""
__version__ = "0.1.0"
