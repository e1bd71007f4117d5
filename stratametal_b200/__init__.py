"""B200-native (sm_100a) implementation of StrataMetal's Mixture-of-Experts block.

The product is the CUDA library ``libsmoe.so`` behind the C ABI in ``include/smoe.h``: router (bf16 GEMV,
softmax, top-k, renormalise), token -> expert dispatch, dequant-fused Q2_0 / IQ2_S expert products with the
sigmoid-gated shared expert, and the weighted combine.  ``api`` is a thin Python front end of that ABI;
``synth`` generates seeded layers in the reference's block formats.
"""
from ._lib import SmoeError, lib, lib_path  # noqa: F401

__version__ = "0.1.0"
