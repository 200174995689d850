// Hessian processing for GPTQ / Qronos (gptq_ref.py:44-93):
//   * act-order permutation (descending diag, stable, gptq_ref.py:67-70);
//   * damping and permutation (gptq_ref.py:72-83);
//   * the upper inverse-Cholesky factor U = chol(Hd^-1, upper).
//
// U is computed without forming Hd^-1: with J the exchange matrix, factor
// J Hd J = L L^T (lower Cholesky), so Hd = R R^T with R = J L J upper, and
// Hd^-1 = (R^-1)^T R^-1, i.e. U = R^-1 = J L^-1 J.  Cost: one blocked
// Cholesky (n^3/3) plus one triangular inverse, all in float32.
//
// Blocked right-looking Cholesky, panel width 128: a single-CTA kernel factors
// the diagonal block in shared memory (flagging a non-positive or non-finite
// pivot in a device status word instead of producing NaNs) and inverts it;
// the panel solve and the trailing rank-64 update are fp32 GEMMs.  The
// triangular inverse is recursive (X21 = -L22^-1 L21 L11^-1) with all 128x128
// diagonal blocks inverted by one batched launch.
#include "gq_common.cuh"

#include <algorithm>
#include <cmath>

namespace gq {

int sgemm(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
          const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int uplo, cudaStream_t st);

// ---------------------------------------------------------------------------
// Act-order permutation by ranking: element i goes to position
// #{j : key_j > key_i} + #{j : key_j == key_i, j > i}.  NaN ranks above
// every number (jnp.argsort sorts NaN last; the reversal puts it first).
__device__ __forceinline__ bool key_gt(float a, float b) {
  bool na = isnan(a), nb = isnan(b);
  if (na || nb) return na && !nb;
  return a > b;
}
__device__ __forceinline__ bool key_eq(float a, float b) {
  bool na = isnan(a), nb = isnan(b);
  if (na || nb) return na && nb;
  return a == b;
}

__global__ void act_order_rank_kernel(const float* __restrict__ h, int64_t d, int64_t ldh,
                                      int32_t* __restrict__ perm) {
  __shared__ float keys[1024];
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  float ki = (i < d) ? h[i * ldh + i] : 0.f;
  int64_t rank = 0;
  for (int64_t base = 0; base < d; base += 1024) {
    int64_t cnt = min((int64_t)1024, d - base);
    __syncthreads();
    for (int64_t t = threadIdx.x; t < cnt; t += blockDim.x) keys[t] = h[(base + t) * ldh + base + t];
    __syncthreads();
    if (i < d) {
      for (int64_t t = 0; t < cnt; ++t) {
        float kj = keys[t];
        int64_t j = base + t;
        rank += key_gt(kj, ki) || (key_eq(kj, ki) && j > i);
      }
    }
  }
  if (i < d) perm[rank] = (int32_t)i;
}

__global__ void iota_kernel(int32_t* perm, int64_t d) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < d) perm[i] = (int32_t)i;
}

int act_order_perm(const float* h, int64_t d, int64_t ldh, int ordering, int32_t* perm,
                   cudaStream_t st) {
  if (d == 0) return GQ_OK;
  unsigned blocks = (unsigned)ceil_div(d, 256);
  if (ordering == 0) iota_kernel<<<blocks, 256, 0, st>>>(perm, d);
  else act_order_rank_kernel<<<blocks, 256, 0, st>>>(h, d, ldh, perm);
  return check_launch("gq_act_order_perm");
}

// ---------------------------------------------------------------------------
// mean(diag(h)) in float32 (order-independent of the permutation); 0 -> 1.
__global__ void diag_mean_kernel(const float* __restrict__ h, int64_t d, int64_t ldh,
                                 float* __restrict__ out) {
  __shared__ float part[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < d; i += blockDim.x) s += h[i * ldh + i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = (threadIdx.x < (blockDim.x >> 5)) ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) {
      float mean = v / (float)d;
      out[0] = (mean == 0.f) ? 1.f : mean;
    }
  }
}

// ht[i][j] = h[p[n-1-i]][p[n-1-j]] + damp * mean * (i == j)   (reversed order)
// hd[i][j] = h[p[i]][p[j]] + damp * mean * (i == j)            (optional)
__global__ void damp_permute_kernel(const float* __restrict__ h, int64_t n, int64_t ldh,
                                    const int32_t* __restrict__ perm, const float* __restrict__ mean,
                                    float damp, float* __restrict__ ht, float* __restrict__ hd) {
  int64_t i = blockIdx.y;
  float dv = damp * mean[0];
  int64_t pi_rev = perm ? perm[n - 1 - i] : (n - 1 - i);
  int64_t pi = perm ? perm[i] : i;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x) {
    int64_t pj_rev = perm ? perm[n - 1 - j] : (n - 1 - j);
    float v = h[pi_rev * ldh + pj_rev];
    if (i == j) v = v + dv;
    ht[i * n + j] = v;
    if (hd) {
      int64_t pj = perm ? perm[j] : j;
      float w = h[pi * ldh + pj];
      if (i == j) w = w + dv;
      hd[i * n + j] = w;
    }
  }
}

// ---------------------------------------------------------------------------
// Diagonal blocks of NB x NB are factored and inverted by one 1024-thread CTA
// with the block held in registers: thread (ty, tx) of a 32 x 32 grid owns the
// 4 x 4 tile rows 4ty..4ty+3, columns 4tx..4tx+3.  Each elimination step
// publishes one column (and for the inverse one row) through double-buffered
// shared memory, so a step costs one barrier, eight shared loads and sixteen
// register FMAs per thread; warps whose tiles are finished skip the update.
constexpr int NB = 128;
constexpr int DIAG_THREADS = 1024;
constexpr size_t DIAG_SMEM = 0;

// Lower Cholesky of v (the kb x kb block; identity beyond kb), in place.  A
// pivot that is not > 0 (or not finite) sets *bad and continues with 1.
__device__ void chol_regs(float (&v)[4][4], int kb, int* bad, float (*colbuf)[NB]) {
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int j = 0; j < NB; ++j) {
    float* col = colbuf[j & 1];
    if (tx == (j >> 2)) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (t == (j & 3)) col[4 * ty + i] = v[i][t];
    }
    __syncthreads();
    float djj = col[j];
    if (j < kb && (!(djj > 0.f) || !isfinite(djj))) {
      if (threadIdx.x == 0) *bad = 1;
      djj = 1.f;
    }
    if (j >= kb) djj = 1.f;
    const float ljj = sqrtf(djj);
    const float rinv = 1.f / djj;
    if (4 * ty + 3 > j && 4 * tx + 3 > j && 4 * tx <= 4 * ty + 3) {
      // trailing update s[r][c] -= s[r][j] s[c][j] / s[j][j] for j < c <= r
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = 4 * ty + i;
        const float srj = col[r] * rinv;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int c = 4 * tx + t;
          if (c > j && c <= r) v[i][t] = fmaf(-srj, col[c], v[i][t]);
        }
      }
    }
    if (tx == (j >> 2)) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = 4 * ty + i;
        const float lv = (r == j) ? ljj : col[r] / ljj;
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (t == (j & 3) && r >= j) v[i][t] = lv;
      }
    }
  }
}

// x = L^-1 for the lower L in v (right-looking substitution on x = I): step k
// scales row k by 1 / L[k][k] and removes it from the rows below.
__device__ void trinv_regs(const float (&v)[4][4], float (&x)[4][4], float (*colbuf)[NB],
                           float (*rowbuf)[NB]) {
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int t = 0; t < 4; ++t) x[i][t] = (4 * ty + i == 4 * tx + t) ? 1.f : 0.f;
  for (int k = 0; k < NB; ++k) {
    float* col = colbuf[k & 1];
    float* row = rowbuf[k & 1];
    if (tx == (k >> 2)) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (t == (k & 3)) col[4 * ty + i] = v[i][t];
    }
    if (ty == (k >> 2)) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (i == (k & 3)) row[4 * tx + t] = x[i][t];
    }
    __syncthreads();
    const float rk = 1.f / col[k];
    if (4 * ty + 3 > k && 4 * tx <= k) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = 4 * ty + i;
        const float lrk = col[r];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int c = 4 * tx + t;
          if (r > k && c <= k) x[i][t] = fmaf(-lrk, row[c] * rk, x[i][t]);
        }
      }
    }
    if (ty == (k >> 2)) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (i == (k & 3)) x[i][t] *= rk;
    }
  }
}

// Cholesky of the kb x kb lower block at a (ld lda) in place (strict upper
// part zeroed) and its inverse into inv (NB x NB, ld NB, zero padded).
__global__ void __launch_bounds__(DIAG_THREADS)
potrf_diag_kernel(float* __restrict__ a, int64_t lda, int kb, float* __restrict__ inv,
                  int* __restrict__ status) {
  __shared__ float colbuf[2][NB];
  __shared__ float rowbuf[2][NB];
  __shared__ int bad;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  if (threadIdx.x == 0) bad = 0;
  float v[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int r = 4 * ty + i, c = 4 * tx + t;
      v[i][t] = (r < kb && c < kb) ? ((c <= r) ? a[r * lda + c] : 0.f) : ((r == c) ? 1.f : 0.f);
    }
  __syncthreads();
  chol_regs(v, kb, &bad, colbuf);
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int r = 4 * ty + i, c = 4 * tx + t;
      if (r < kb && c < kb) a[r * lda + c] = (c <= r) ? v[i][t] : 0.f;
    }
  float x[4][4];
  __syncthreads();
  trinv_regs(v, x, colbuf, rowbuf);
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int r = 4 * ty + i, c = 4 * tx + t;
      inv[r * NB + c] = (r < kb && c < kb && c <= r) ? x[i][t] : 0.f;
    }
  __syncthreads();
  if (threadIdx.x == 0 && bad) atomicExch(status, GQ_DEVERR_NOTPD);
}

// Batched in-place inverse of the NB x NB lower-triangular diagonal blocks of a.
__global__ void __launch_bounds__(DIAG_THREADS)
trinv_diag_blocks_kernel(float* __restrict__ a, int64_t n, int64_t lda) {
  __shared__ float colbuf[2][NB];
  __shared__ float rowbuf[2][NB];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int64_t b0 = (int64_t)blockIdx.x * NB;
  const int kb = (int)min((int64_t)NB, n - b0);
  float v[4][4], x[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int r = 4 * ty + i, c = 4 * tx + t;
      v[i][t] = (r < kb && c < kb) ? ((c <= r) ? a[(b0 + r) * lda + b0 + c] : 0.f)
                                   : ((r == c) ? 1.f : 0.f);
    }
  trinv_regs(v, x, colbuf, rowbuf);
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int r = 4 * ty + i, c = 4 * tx + t;
      if (r < kb && c < kb) a[(b0 + r) * lda + b0 + c] = (c <= r) ? x[i][t] : 0.f;
    }
}

// Zero the strict upper triangle of an n x n matrix (ld).
__global__ void zero_upper_kernel(float* __restrict__ a, int64_t n, int64_t lda) {
  int64_t r = blockIdx.y;
  for (int64_t c = r + 1 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < n;
       c += (int64_t)gridDim.x * blockDim.x)
    a[r * lda + c] = 0.f;
}

// u[i][j] = linv[n-1-i][n-1-j]
__global__ void reverse_copy_kernel(const float* __restrict__ linv, int64_t n, int64_t ldl,
                                    float* __restrict__ u, int64_t ldu) {
  int64_t i = blockIdx.y;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x)
    u[i * ldu + j] = linv[(n - 1 - i) * ldl + (n - 1 - j)];
}

// Blocked lower Cholesky of a (n x n, ld n) in place; panel scratch p (n x NB),
// diagonal-inverse scratch dinv (NB x NB).
int cholesky_lower(float* a, int64_t n, float* p, float* dinv, int* status, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    GQ_CHECK_CUDA(cudaFuncSetAttribute(potrf_diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)DIAG_SMEM));
    GQ_CHECK_CUDA(cudaFuncSetAttribute(trinv_diag_blocks_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DIAG_SMEM));
    attr = true;
  }
  for (int64_t k0 = 0; k0 < n; k0 += NB) {
    int kb = (int)std::min<int64_t>(NB, n - k0);
    float* akk = a + k0 * n + k0;
    potrf_diag_kernel<<<1, DIAG_THREADS, DIAG_SMEM, st>>>(akk, n, kb, dinv, status);
    GQ_TRY(check_launch("potrf_diag"));
    int64_t rem = n - k0 - kb;
    if (rem <= 0) break;
    float* a21 = a + (k0 + kb) * n + k0;
    // P = A21 * L11^-T   (rem x kb)
    GQ_TRY(sgemm(0, 1, rem, kb, kb, 1.f, a21, n, dinv, NB, 0.f, p, NB, 0, st));
    // A22 -= P P^T (lower tiles)
    float* a22 = a + (k0 + kb) * n + (k0 + kb);
    GQ_TRY(sgemm(0, 1, rem, rem, kb, -1.f, p, NB, p, NB, 1.f, a22, n, 1, st));
    GQ_CHECK_CUDA(cudaMemcpy2DAsync(a21, n * sizeof(float), p, NB * sizeof(float),
                                    kb * sizeof(float), rem, cudaMemcpyDeviceToDevice, st));
  }
  return GQ_OK;
}

int transpose2d(const float* src, int64_t rows, int64_t cols, int64_t lds, float* dst, int64_t ldd,
                cudaStream_t st);

// Recursive lower-triangular inverse of a[0:n, 0:n] (ld lda) in place.  The
// NB x NB diagonal blocks must already be inverted; the strict upper triangle
// must be zero.  With [[L11, 0], [L21, L22]]^-1 = [[X11, 0], [X21, X22]],
// X21 = -X22 L21 X11, evaluated as two products whose operands are both
// K-major (tensor-core GEMM path):  Tt = X11^T L21^T,  X21 = -X22 Tt^T.
// scratch: at least (n/2 + 64) * (n + 64) floats.
int trinv_rec(float* a, int64_t n, int64_t lda, float* scratch, cudaStream_t st) {
  if (n <= NB) return GQ_OK;
  int64_t n1 = ((n / 2 + NB - 1) / NB) * NB;
  if (n1 >= n) n1 = n - NB;
  int64_t n2 = n - n1;
  float* a11 = a;
  float* a21 = a + n1 * lda;
  float* a22 = a + n1 * lda + n1;
  GQ_TRY(trinv_rec(a11, n1, lda, scratch, st));
  GQ_TRY(trinv_rec(a22, n2, lda, scratch, st));
  float* s1 = scratch;            // X11^T, n1 x n1
  float* tt = scratch + n1 * n1;  // Tt = (L21 X11)^T, n1 x n2
  GQ_TRY(transpose2d(a11, n1, n1, lda, s1, n1, st));
  GQ_TRY(sgemm(0, 1, n1, n2, n1, 1.f, s1, n1, a21, lda, 0.f, tt, n2, 0, st));
  GQ_TRY(sgemm(0, 1, n2, n1, n2, -1.f, a22, lda, tt, n2, 0.f, a21, lda, 0, st));
  return GQ_OK;
}

int64_t hessian_ws_floats(int64_t d) {
  int64_t half = d / 2 + NB;
  return d * d + d * NB + NB * NB + half * (d + NB) + 64;
}

}  // namespace gq

extern "C" {

int gq_act_order_perm(const float* h, int64_t d, int64_t ldh, int ordering, int32_t* perm,
                      void* stream) {
  GQ_REQUIRE(d >= 0 && ldh >= d, "gq_act_order_perm: bad shape");
  GQ_REQUIRE(ordering == 0 || ordering == 1, "gq_act_order_perm: ordering must be 0 or 1");
  GQ_REQUIRE(d < (1ll << 31), "gq_act_order_perm: d too large");
  return gq::act_order_perm(h, d, ldh, ordering, perm, gq::as_stream(stream));
}

int64_t gq_hessian_factor_workspace_size(int64_t d) {
  return gq::hessian_ws_floats(d) * (int64_t)sizeof(float);
}

int gq_hessian_factor(const float* h, int64_t d, int64_t ldh, const int32_t* perm,
                      double damp_percent, float* u, int64_t ldu, float* hd_out, void* workspace,
                      int64_t workspace_bytes, int* attempt_out, void* stream) {
  GQ_REQUIRE(h != nullptr && u != nullptr, "gq_hessian_factor: NULL h or u");
  GQ_REQUIRE(d > 0 && ldh >= d && ldu >= d, "gq_hessian_factor: bad shape");
  GQ_REQUIRE(workspace_bytes >= gq_hessian_factor_workspace_size(d),
             "gq_hessian_factor: workspace too small (%lld < %lld)", (long long)workspace_bytes,
             (long long)gq_hessian_factor_workspace_size(d));
  GQ_REQUIRE(damp_percent >= 0.0, "gq_hessian_factor: negative damp_percent");
  cudaStream_t st = gq::as_stream(stream);
  float* ws = reinterpret_cast<float*>(workspace);
  float* ht = ws;                                  // d*d
  float* p = ht + d * d;                           // d*64
  float* dinv = p + d * gq::NB;                    // 64*64
  float* scratch = dinv + gq::NB * gq::NB;         // (d/2+64) x (d+64)
  int64_t half = d / 2 + gq::NB;
  float* mean = scratch + half * (d + gq::NB);     // 1 float
  int* status = reinterpret_cast<int*>(mean + 16);  // 1 int

  gq::diag_mean_kernel<<<1, 1024, 0, st>>>(h, d, ldh, mean);
  GQ_TRY(gq::check_launch("diag_mean"));
  for (int attempt = 0; attempt < 5; ++attempt) {
    double damp = std::pow(10.0, attempt) * damp_percent;
    GQ_CHECK_CUDA(cudaMemsetAsync(status, 0, sizeof(int), st));
    dim3 grid((unsigned)std::min<int64_t>(gq::ceil_div(d, 256), 64), (unsigned)d);
    gq::damp_permute_kernel<<<grid, 256, 0, st>>>(h, d, ldh, perm, mean, (float)damp, ht, hd_out);
    GQ_TRY(gq::check_launch("damp_permute"));
    GQ_TRY(gq::cholesky_lower(ht, d, p, dinv, status, st));
    int host_status = 0;
    GQ_CHECK_CUDA(cudaMemcpyAsync(&host_status, status, sizeof(int), cudaMemcpyDeviceToHost, st));
    GQ_CHECK_CUDA(cudaStreamSynchronize(st));
    if (host_status != gq::GQ_DEVERR_NONE) continue;
    // L^-1 in place, then U = J L^-1 J
    dim3 gz((unsigned)std::min<int64_t>(gq::ceil_div(d, 256), 64), (unsigned)d);
    gq::zero_upper_kernel<<<gz, 256, 0, st>>>(ht, d, d);
    GQ_TRY(gq::check_launch("zero_upper"));
    gq::trinv_diag_blocks_kernel<<<(unsigned)gq::ceil_div(d, gq::NB), gq::DIAG_THREADS,
                                   gq::DIAG_SMEM, st>>>(ht, d, d);
    GQ_TRY(gq::check_launch("trinv_diag_blocks"));
    GQ_TRY(gq::trinv_rec(ht, d, d, scratch, st));
    dim3 g2((unsigned)std::min<int64_t>(gq::ceil_div(d, 256), 64), (unsigned)d);
    gq::reverse_copy_kernel<<<g2, 256, 0, st>>>(ht, d, d, u, ldu);
    GQ_TRY(gq::check_launch("reverse_copy"));
    if (attempt_out) *attempt_out = attempt;
    return GQ_OK;
  }
  if (attempt_out) *attempt_out = -1;
  return gq::fail(GQ_ENOTPD, "gq_hessian_factor: damped Hessian not positive definite after 5 attempts");
}

}  // extern "C"
