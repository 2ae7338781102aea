// Float32 linspace positions of the reference's compressed keys, bit-exact on the device.
//
// The reference places compressed key i of a sequence of T tokens at
// torch.linspace(0, T-1, n_cmp)[i] (float32; nsa_reference.py:35, 62) and uses that position
// both to map the key to a selection block (floor division by l_prime, :36) and as its causal
// position in the compressed branch (cpos <= t, :63).  PyTorch's CPU kernel rounds the step to
// float32 and forms each value in double from the nearer end of the range before rounding; the
// floor division follows PyTorch's float floor-divide.  The _rn intrinsics keep the compiler
// from contracting the products into FMAs, which would change the rounding.
#pragma once
#include <math.h>

namespace nsa {

__device__ __forceinline__ float linspace_f32(int i, int T, int n) {
  if (n == 1) return 0.f;
  const float step = __fdiv_rn((float)(T - 1), (float)(n - 1));
  if (i < n / 2) return (float)__dmul_rn((double)step, (double)i);
  return (float)__dsub_rn((double)(T - 1), __dmul_rn((double)step, (double)(n - 1 - i)));
}

__device__ __forceinline__ float floor_div_f32(float a, float b) {
  const float mod = fmodf(a, b);
  float div = __fdiv_rn(__fsub_rn(a, mod), b);
  if (mod != 0.f && ((b < 0.f) != (mod < 0.f))) div = __fsub_rn(div, 1.f);
  if (div != 0.f) {
    float fl = floorf(div);
    if (__fsub_rn(div, fl) > 0.5f) fl = __fadd_rn(fl, 1.f);
    return fl;
  }
  return copysignf(0.f, __fdiv_rn(a, b));
}

// Last compressed key visible to query t (the largest i with linspace(i) <= t; the positions are
// non-decreasing and linspace(0) = 0, so it is >= 0 for t >= 0).
__device__ __forceinline__ int compressed_limit(int t, int T, int n) {
  if (n <= 1) return n - 1;
  const int est = (int)floor((double)t * (double)(n - 1) / (double)(T - 1));
  int best = -1;
  for (int i = max(0, est - 2); i <= min(n - 1, est + 3); ++i)
    if (linspace_f32(i, T, n) <= (float)t) best = i;
  return best;
}

}  // namespace nsa
