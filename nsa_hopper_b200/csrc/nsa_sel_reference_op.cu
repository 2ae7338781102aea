// Drop-in source for harnesses written against the reference's JIT build, e.g.
//   mod = torch.utils.cpp_extension.load('nsa_v2', ['<this file>'],
//                                        extra_cuda_cflags=['-arch=sm_90a', '-O3', ...])
//   O = mod.forward(Q, K, V, sel, l_prime, BQ, cyc)
// (reference test_v2.py:4-6, 22).  It holds no device code: it compiles the PyTorch binding,
// which forwards to the prebuilt sm_100a library libnsa_sel.so next to the package sources.
#include "nsa_sel_torch.cpp"
