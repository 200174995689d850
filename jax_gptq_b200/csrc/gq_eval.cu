// Masked next-token negative log-likelihood for perplexity evaluation -- the
// computation of eval.py:9-22 (_masked_nll_from_logits).
//
// For every batch entry b and position t < T - 1 the prediction at t is scored
// against the label at t + 1: nll = logsumexp(logits[b, t, :]) -
// logits[b, t, label[b, t + 1]], and positions whose label is -100 contribute
// nothing and are not counted (eval.py:11-20).  Labels outside [0, V) are
// clamped to the range, as JAX clamps out-of-range gathers.
//
// One CTA per scored position reads its V logits once (16-byte loads when the
// row is aligned), so the kernel is HBM-bound: 4 (fp32) or 2 (bf16) bytes per
// logit.  Each position's nll goes to row_nll in float64; a second one-CTA
// kernel adds them in a fixed order, so the sum is deterministic.
#include "gq_common.cuh"

#include <cuda_bf16.h>

namespace gq {
namespace evalk {

constexpr int THREADS = 256;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float x = (l < THREADS / 32) ? red[l] : -INFINITY;
    x = warp_max(x);
    if (l == 0) red[0] = x;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ double block_sum_d(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  double r = 0.0;
  if (threadIdx.x == 0)
    for (int i = 0; i < THREADS / 32; ++i) r += red[i];  // fixed order
  return r;  // valid in thread 0
}

// Loads 4 consecutive logits starting at element e (e % 4 == 0 when vec).
template <typename T>
__device__ __forceinline__ void load4(const T* row, int64_t e, float (&x)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* row, int64_t e, float (&x)[4]) {
  const float4 v = __ldg(reinterpret_cast<const float4*>(row + e));
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* row, int64_t e,
                                                     float (&x)[4]) {
  const uint2 v = __ldg(reinterpret_cast<const uint2*>(row + e));
  x[0] = __uint_as_float(v.x << 16);
  x[1] = __uint_as_float(v.x & 0xffff0000u);
  x[2] = __uint_as_float(v.y << 16);
  x[3] = __uint_as_float(v.y & 0xffff0000u);
}

template <typename T>
__global__ void __launch_bounds__(THREADS) masked_nll_kernel(const T* __restrict__ logits,
                                                             int64_t T_len, int64_t V,
                                                             const int64_t* __restrict__ labels,
                                                             double* __restrict__ row_nll,
                                                             int* __restrict__ row_mask) {
  __shared__ float redf[THREADS / 32];
  __shared__ double redd[THREADS / 32];
  const int64_t r = blockIdx.x;  // scored position: b * (T - 1) + t
  const int64_t b = r / (T_len - 1), t = r % (T_len - 1);
  const int64_t lab = labels[b * T_len + t + 1];
  if (lab == -100) {  // uniform across the CTA: nothing to read
    if (threadIdx.x == 0) {
      row_nll[r] = 0.0;
      row_mask[r] = 0;
    }
    return;
  }
  const T* row = logits + (b * T_len + t) * V;
  const bool vec = (reinterpret_cast<uintptr_t>(row) % (4 * sizeof(T))) == 0;
  const int64_t v4 = vec ? (V / 4) * 4 : 0;
  float mx = -INFINITY;
  for (int64_t e = 4 * (int64_t)threadIdx.x; e < v4; e += 4 * THREADS) {
    float x[4];
    load4<T>(row, e, x);
    mx = fmaxf(mx, fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])));
  }
  for (int64_t e = v4 + threadIdx.x; e < V; e += THREADS) mx = fmaxf(mx, to_f<T>(row[e]));
  mx = block_max(mx, redf);
  // sum of exp(x - max): per-thread float partial sums (each term <= 1), the
  // cross-thread sum in double
  float acc = 0.f;
  for (int64_t e = 4 * (int64_t)threadIdx.x; e < v4; e += 4 * THREADS) {
    float x[4];
    load4<T>(row, e, x);
    acc += expf(x[0] - mx) + expf(x[1] - mx) + expf(x[2] - mx) + expf(x[3] - mx);
  }
  for (int64_t e = v4 + threadIdx.x; e < V; e += THREADS) acc += expf(to_f<T>(row[e]) - mx);
  const double s = block_sum_d((double)acc, redd);
  if (threadIdx.x == 0) {
    const int64_t li = lab < 0 ? 0 : (lab >= V ? V - 1 : lab);
    const double lse = (double)mx + log(s);
    row_nll[r] = lse - (double)to_f<T>(row[li]);
    row_mask[r] = 1;
  }
}

// Fixed-order sum of row_nll and count of scored positions: thread i adds
// rows i, i + 1024, ... in order, then thread 0 adds the 1024 partials in order.
__global__ void __launch_bounds__(1024) nll_reduce_kernel(const double* __restrict__ row_nll,
                                                          const int* __restrict__ row_mask,
                                                          int64_t rows, double* nll_sum,
                                                          int64_t* count) {
  __shared__ double ps[1024];
  __shared__ long long pc[1024];
  double s = 0.0;
  long long c = 0;
  for (int64_t i = threadIdx.x; i < rows; i += 1024) {
    s += row_nll[i];
    c += row_mask[i];
  }
  ps[threadIdx.x] = s;
  pc[threadIdx.x] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    double ts = 0.0;
    long long tc = 0;
    for (int i = 0; i < 1024; ++i) {
      ts += ps[i];
      tc += pc[i];
    }
    *nll_sum = ts;
    *count = tc;
  }
}

}  // namespace evalk
}  // namespace gq

extern "C" {

int64_t gq_masked_nll_workspace_size(int64_t batch, int64_t tokens) {
  if (batch <= 0 || tokens <= 1) return 256;
  const int64_t rows = batch * (tokens - 1);
  return ((rows * 8 + 255) & ~int64_t(255)) + rows * 4 + 256;
}

int gq_masked_nll(const void* logits, int dtype, int64_t batch, int64_t tokens, int64_t vocab,
                  const int64_t* labels, double* nll_sum, int64_t* count, void* workspace,
                  int64_t workspace_bytes, void* stream) {
  GQ_REQUIRE(dtype == 0 || dtype == 1, "gq_masked_nll: dtype must be 0 (float32) or 1 (bf16)");
  GQ_REQUIRE(batch >= 0 && tokens >= 0 && vocab >= 1, "gq_masked_nll: bad shape");
  GQ_REQUIRE(nll_sum != nullptr && count != nullptr, "gq_masked_nll: NULL output");
  GQ_REQUIRE(workspace_bytes >= gq_masked_nll_workspace_size(batch, tokens),
             "gq_masked_nll: workspace too small");
  GQ_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
             "gq_masked_nll: workspace must be 256-byte aligned");
  cudaStream_t st = gq::as_stream(stream);
  const int64_t rows = (batch > 0 && tokens > 1) ? batch * (tokens - 1) : 0;
  GQ_REQUIRE(rows <= 0x7fffffffll, "gq_masked_nll: too many positions");
  GQ_REQUIRE(rows == 0 || (logits != nullptr && labels != nullptr), "gq_masked_nll: NULL input");
  double* row_nll = reinterpret_cast<double*>(workspace);
  int* row_mask = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) +
                                         ((rows * 8 + 255) & ~int64_t(255)));
  if (rows > 0) {
    if (dtype == 0)
      gq::evalk::masked_nll_kernel<float><<<(unsigned)rows, gq::evalk::THREADS, 0, st>>>(
          static_cast<const float*>(logits), tokens, vocab, labels, row_nll, row_mask);
    else
      gq::evalk::masked_nll_kernel<__nv_bfloat16><<<(unsigned)rows, gq::evalk::THREADS, 0, st>>>(
          static_cast<const __nv_bfloat16*>(logits), tokens, vocab, labels, row_nll, row_mask);
    GQ_TRY(gq::check_launch("masked_nll"));
  }
  gq::evalk::nll_reduce_kernel<<<1, 1024, 0, st>>>(row_nll, row_mask, rows, nll_sum, count);
  return gq::check_launch("nll_reduce");
}

}  // extern "C"
