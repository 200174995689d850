// RTN quantize/dequantize (quant.py:6-37) with an optional column
// permutation (gptq_ref.py:152-155).  HBM-bound: one CTA per row; the row is
// read once, coalesced, into shared memory, groups are formed in permuted
// order by a shared-memory gather, and dequantized values / codes are written
// back in original column order, again coalesced.
#include "gq_common.cuh"
#include "gq_quant.cuh"

namespace gq {

constexpr int kRtnThreads = 256;

// Shared layout: row values (n floats, original order; overwritten in place
// by the dequantized values), codes (n bytes), then per-group scale and zero.
__global__ void __launch_bounds__(kRtnThreads)
rtn_row_kernel(const float* __restrict__ w, int64_t n, int64_t ldw,
               const int32_t* __restrict__ perm, int group_size, QParams qp, int sym,
               float* __restrict__ dequant, uint8_t* __restrict__ codes,
               float* __restrict__ scales, float* __restrict__ zeros) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int64_t row = blockIdx.x;
  const int64_t n_groups = n / group_size;
  float* srow = reinterpret_cast<float*>(smem);
  float* sscale = srow + n;
  float* szero = sscale + n_groups;
  uint8_t* scode = reinterpret_cast<uint8_t*>(szero + n_groups);

  const float* wr = w + row * ldw;
  const bool vec = ((reinterpret_cast<uintptr_t>(wr) & 15) == 0) && (n % 4 == 0);
  if (vec) {
    const float4* w4 = reinterpret_cast<const float4*>(wr);
    float4* s4 = reinterpret_cast<float4*>(srow);
    for (int64_t c = threadIdx.x; c < n / 4; c += blockDim.x) s4[c] = w4[c];
  } else {
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) srow[c] = wr[c];
  }
  __syncthreads();

  // Phase 1: one warp per group (permuted order) -> scale / zero.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int64_t gi = warp; gi < n_groups; gi += nwarps) {
    float mn = INFINITY, mx = -INFINITY, ma = 0.f;
    for (int e = lane; e < group_size; e += 32) {
      int64_t j = gi * group_size + e;
      float v = srow[perm ? perm[j] : j];
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
      ma = fmaxf(ma, fabsf(v));
    }
    mn = warp_min(mn);
    mx = warp_max(mx);
    ma = warp_max(ma);
    if (lane == 0) {
      float s, z;
      if (sym) group_scale_zero(-ma, ma, qp, sym, s, z);
      else group_scale_zero(mn, mx, qp, sym, s, z);
      sscale[gi] = s;
      szero[gi] = z;
    }
  }
  __syncthreads();

  // Phase 2: quantize every element; permuted position j lives at srow[perm[j]].
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
    int64_t c = perm ? perm[j] : j;
    int64_t gi = j / group_size;
    float dq;
    float q = quantize_one(srow[c], sscale[gi], szero[gi], qp, dq);
    srow[c] = dq;
    scode[c] = (uint8_t)(int)(q - qp.qmin);
  }
  __syncthreads();

  // Phase 3: coalesced write-back in original order.
  if (dequant) {
    float* dr = dequant + row * n;
    if (n % 4 == 0) {
      float4* d4 = reinterpret_cast<float4*>(dr);
      const float4* s4 = reinterpret_cast<const float4*>(srow);
      for (int64_t c = threadIdx.x; c < n / 4; c += blockDim.x) d4[c] = s4[c];
    } else {
      for (int64_t c = threadIdx.x; c < n; c += blockDim.x) dr[c] = srow[c];
    }
  }
  if (codes) {
    uint8_t* cr = codes + row * n;
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) cr[c] = scode[c];
  }
  if (scales) {
    for (int64_t gi = threadIdx.x; gi < n_groups; gi += blockDim.x) {
      scales[row * n_groups + gi] = sscale[gi];
    }
  }
  if (zeros) {
    for (int64_t gi = threadIdx.x; gi < n_groups; gi += blockDim.x) {
      zeros[row * n_groups + gi] = szero[gi];
    }
  }
}

size_t rtn_smem_bytes(int64_t n, int group_size) {
  int64_t n_groups = n / group_size;
  return (size_t)(n * 4 + n_groups * 8 + n + 16);
}

int rtn_launch(const float* w, int64_t m, int64_t n, int64_t ldw, const int32_t* perm,
               int w_bits, int group_size, int sym, float* dequant, uint8_t* codes,
               float* scales, float* zeros, cudaStream_t st) {
  size_t smem = rtn_smem_bytes(n, group_size);
  if (smem > 220 * 1024)
    return fail(GQ_EUNSUPPORTED, "gq_rtn: row of %lld columns exceeds the shared-memory row buffer",
                (long long)n);
  if (m == 0 || n == 0) return GQ_OK;
  GQ_CHECK_CUDA(cudaFuncSetAttribute(rtn_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
  QParams qp = make_qparams(w_bits, sym);
  rtn_row_kernel<<<(unsigned)m, kRtnThreads, smem, st>>>(w, n, ldw, perm, group_size, qp, sym,
                                                         dequant, codes, scales, zeros);
  return check_launch("gq_rtn");
}

int check_quant_args(const char* who, int64_t m, int64_t n, int w_bits, int group_size, int sym) {
  GQ_REQUIRE(m >= 0 && n >= 0, "%s: negative shape", who);
  GQ_REQUIRE(group_size > 0 && n % group_size == 0,
             "%s: group_size must be positive and divide in_features exactly", who);
  GQ_REQUIRE(w_bits >= (sym ? 2 : 1) && w_bits <= 8, "%s: w_bits=%d outside [%d, 8]", who, w_bits,
             sym ? 2 : 1);
  return GQ_OK;
}

}  // namespace gq

extern "C" int gq_rtn(const float* w, int64_t m, int64_t n, int64_t ldw, const int32_t* perm,
                      int w_bits, int group_size, int sym, float* dequant, uint8_t* codes,
                      float* scales, float* zeros, void* stream) {
  GQ_TRY(gq::check_quant_args("gq_rtn", m, n, w_bits, group_size, sym));
  GQ_REQUIRE(w != nullptr || m * n == 0, "gq_rtn: w is NULL");
  GQ_REQUIRE(ldw >= n, "gq_rtn: ldw < n");
  return gq::rtn_launch(w, m, n, ldw, perm, w_bits, group_size, sym, dequant, codes, scales, zeros,
                        gq::as_stream(stream));
}
