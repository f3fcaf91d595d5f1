"""B200-native DFA-restricted output head for SmolLM2-135M (market_sim).

The product is ``libmfhead.so`` (CUDA kernels for sm_100a behind the C-ABI
of ``include/mf_head.h``) plus the C++ ``marketforge::cuda`` wrapper
``libmarketforge_b200.so``.  ``market_sim_b200.head`` mirrors the
reference's head interface in Python over the same C-ABI.
"""
__all__ = ["head", "synth", "build"]
