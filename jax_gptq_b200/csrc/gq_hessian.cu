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
// Blocked right-looking Cholesky, panel width 64: a single-CTA kernel factors
// the diagonal block in shared memory (flagging a non-positive or non-finite
// pivot in a device status word instead of producing NaNs) and inverts it;
// the panel solve and the trailing rank-64 update are fp32 GEMMs.  The
// triangular inverse is recursive (X21 = -L22^-1 L21 L11^-1) with all 64x64
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
// Diagonal block: Cholesky of the kb x kb lower block at a (ld), in place,
// plus its lower-triangular inverse into inv (ld 64, upper part zeroed).
// A pivot that is not > 0 (or not finite) sets *status = GQ_DEVERR_NOTPD.
constexpr int NB = 64;

__global__ void __launch_bounds__(256)
potrf_diag_kernel(float* __restrict__ a, int64_t lda, int kb, float* __restrict__ inv,
                  int* __restrict__ status) {
  __shared__ float s[NB][NB + 1];
  __shared__ float sinv[NB][NB + 1];
  __shared__ int bad;
  const int tid = threadIdx.x;
  if (tid == 0) bad = 0;
  for (int e = tid; e < NB * NB; e += blockDim.x) {
    int r = e / NB, c = e % NB;
    s[r][c] = (r < kb && c < kb && c <= r) ? a[r * lda + c] : ((r == c) ? 1.f : 0.f);
  }
  __syncthreads();
  for (int j = 0; j < kb; ++j) {
    float djj = s[j][j];
    if (!(djj > 0.f) || !isfinite(djj)) {
      if (tid == 0) bad = 1;
      djj = 1.f;  // keep going with a harmless value; the status word reports it
    }
    float ljj = sqrtf(djj);
    __syncthreads();
    if (tid == 0) s[j][j] = ljj;
    for (int r = j + 1 + tid; r < kb; r += blockDim.x) s[r][j] = s[r][j] / ljj;
    __syncthreads();
    // trailing update of the lower part: s[r][c] -= s[r][j] * s[c][j] for j < c <= r
    int rem = kb - j - 1;
    for (int e = tid; e < rem * rem; e += blockDim.x) {
      int r = j + 1 + e / rem, c = j + 1 + e % rem;
      if (c <= r) s[r][c] = fmaf(-s[r][j], s[c][j], s[r][c]);
    }
    __syncthreads();
  }
  // write L back (lower part only) and zero the strict upper part
  for (int e = tid; e < kb * kb; e += blockDim.x) {
    int r = e / kb, c = e % kb;
    a[r * lda + c] = (c <= r) ? s[r][c] : 0.f;
  }
  // inverse by forward substitution, one column per thread
  if (tid < NB) {
    int c = tid;
    for (int r = 0; r < NB; ++r) {
      float v;
      if (r < c) v = 0.f;
      else {
        float acc = (r == c) ? 1.f : 0.f;
        for (int k = c; k < r; ++k) acc = fmaf(-s[r][k], sinv[k][c], acc);
        v = acc / s[r][r];
      }
      sinv[r][c] = v;
    }
  }
  __syncthreads();
  for (int e = tid; e < NB * NB; e += blockDim.x) {
    int r = e / NB, c = e % NB;
    inv[r * NB + c] = (r < kb && c < kb) ? sinv[r][c] : 0.f;
  }
  if (tid == 0 && bad) atomicExch(status, GQ_DEVERR_NOTPD);
}

// Batched lower-triangular inverse of the 64x64 diagonal blocks of a (in place).
__global__ void __launch_bounds__(256) trinv_diag_blocks_kernel(float* __restrict__ a, int64_t n,
                                                                int64_t lda) {
  __shared__ float s[NB][NB + 1];
  __shared__ float sinv[NB][NB + 1];
  const int64_t b0 = (int64_t)blockIdx.x * NB;
  const int kb = (int)min((int64_t)NB, n - b0);
  const int tid = threadIdx.x;
  for (int e = tid; e < NB * NB; e += blockDim.x) {
    int r = e / NB, c = e % NB;
    s[r][c] = (r < kb && c < kb && c <= r) ? a[(b0 + r) * lda + b0 + c] : ((r == c) ? 1.f : 0.f);
  }
  __syncthreads();
  if (tid < NB) {
    int c = tid;
    for (int r = 0; r < NB; ++r) {
      float v;
      if (r < c) v = 0.f;
      else {
        float acc = (r == c) ? 1.f : 0.f;
        for (int k = c; k < r; ++k) acc = fmaf(-s[r][k], sinv[k][c], acc);
        v = acc / s[r][r];
      }
      sinv[r][c] = v;
    }
  }
  __syncthreads();
  for (int e = tid; e < kb * kb; e += blockDim.x) {
    int r = e / kb, c = e % kb;
    a[(b0 + r) * lda + b0 + c] = sinv[r][c];
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

// Blocked lower Cholesky of a (n x n, ld n) in place; panel scratch p (n x 64),
// diagonal-inverse scratch dinv (64 x 64).
int cholesky_lower(float* a, int64_t n, float* p, float* dinv, int* status, cudaStream_t st) {
  for (int64_t k0 = 0; k0 < n; k0 += NB) {
    int kb = (int)std::min<int64_t>(NB, n - k0);
    float* akk = a + k0 * n + k0;
    potrf_diag_kernel<<<1, 256, 0, st>>>(akk, n, kb, dinv, status);
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

// Recursive lower-triangular inverse of a[0:n, 0:n] (ld lda) in place.  The
// 64x64 diagonal blocks must already be inverted; the strict upper triangle
// must be zero.  scratch: at least (n/2 + 64) * (n/2 + 64) floats.
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
  // T = L21 * L11^-1  (n2 x n1)
  GQ_TRY(sgemm(0, 0, n2, n1, n1, 1.f, a21, lda, a11, lda, 0.f, scratch, n1, 0, st));
  // X21 = -L22^-1 * T
  GQ_TRY(sgemm(0, 0, n2, n1, n2, -1.f, a22, lda, scratch, n1, 0.f, a21, lda, 0, st));
  return GQ_OK;
}

int64_t hessian_ws_floats(int64_t d) {
  int64_t half = d / 2 + NB;
  return d * d + d * NB + NB * NB + half * half + 64;
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
  float* scratch = dinv + gq::NB * gq::NB;         // (d/2+64)^2
  int64_t half = d / 2 + gq::NB;
  float* mean = scratch + half * half;             // 1 float
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
    gq::trinv_diag_blocks_kernel<<<(unsigned)gq::ceil_div(d, gq::NB), 256, 0, st>>>(ht, d, d);
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
