"""B200-native (sm_100a) NSA selected-branch attention forward.

The hot path is one CUDA kernel family behind the C ABI in include/nsa_sel.h
(``libnsa_sel.so``, bound by :mod:`nsa_hopper_b200.capi`) and a PyTorch extension
(:mod:`nsa_hopper_b200.ops`) with the reference's op signature
``forward(Q, K, V, sel, l_prime, BQ, cyc)``.  There is no CPU or PyTorch fallback: the ops
raise when the compiled libraries are missing.
"""
__version__ = "1.0.0"
