// Round-to-nearest group quantization arithmetic, shared by the RTN and
// GPTQ-sweep kernels.  Follows src/jax_gptq/quant.py:12-37 operation by
// operation in float32 with explicit round-to-nearest intrinsics so that no
// multiply-add contraction or reciprocal substitution can change a code:
//   asym: scale = max((mx - mn) / qmax, 1e-8); zero = clip(rint(-mn / scale), 0, qmax)
//   sym:  scale = max(max|w| / qmax, 1e-8);    zero = 0
//   q = clip(rint(w / scale + zero), qmin, qmax); dequant = (q - zero) * scale
// rintf rounds half to even, like jnp.round.
#pragma once

#include <cuda_runtime.h>

namespace gq {

struct QParams {
  float qmin, qmax;
};

__host__ __device__ inline QParams make_qparams(int w_bits, int sym) {
  QParams p;
  if (sym) {
    p.qmax = (float)((1 << (w_bits - 1)) - 1);
    p.qmin = -p.qmax;
  } else {
    p.qmax = (float)((1 << w_bits) - 1);
    p.qmin = 0.f;
  }
  return p;
}

// quant.py:23-31.  For sym, pass mn = -max|w| and mx = max|w| (only mx is used).
__device__ __forceinline__ void group_scale_zero(float mn, float mx, QParams p, int sym,
                                                 float& scale, float& zero) {
  if (sym) {
    scale = fmaxf(__fdiv_rn(mx, p.qmax), 1e-8f);
    zero = 0.f;
  } else {
    scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), p.qmax), 1e-8f);
    float z = rintf(__fdiv_rn(-mn, scale));
    zero = fminf(fmaxf(z, 0.f), p.qmax);
  }
}

// quant.py:36-37; returns q (as float) and writes the dequantized value.
__device__ __forceinline__ float quantize_one(float w, float scale, float zero, QParams p,
                                              float& dq) {
  float q = rintf(__fadd_rn(__fdiv_rn(w, scale), zero));
  q = fminf(fmaxf(q, p.qmin), p.qmax);
  dq = __fmul_rn(__fsub_rn(q, zero), scale);
  return q;
}

}  // namespace gq
