// Hessian processing for GPTQ / Qronos (gptq_ref.py:44-93):
//   * act-order permutation (descending diag, stable, gptq_ref.py:67-70);
//   * damping and permutation (gptq_ref.py:72-83);
//   * the upper inverse-Cholesky factor U = chol(Hd^-1, upper).
//
// U is computed without forming Hd^-1: with J the exchange matrix, factor
// J Hd J = L L^T (lower Cholesky), so Hd = R R^T with R = J L J upper, and
// Hd^-1 = (R^-1)^T R^-1, i.e. U = R^-1 = J L^-1 J.  Cost: n^3/3 for the
// Cholesky plus n^3/3 for the triangular inverse, all in float32.
//
// L^-1 is computed by one recursion that interleaves both (inv_chol_rec):
// its leaves are 128 x 128 diagonal blocks, factored and inverted by a
// single-CTA kernel in shared memory (a non-positive or non-finite pivot sets
// a device status word instead of producing NaNs); everything else is fp32
// tensor-core GEMMs whose K is half the current size.
#include "gq_common.cuh"

#include <algorithm>
#include <cmath>

namespace gq {

int sgemm(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
          const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int uplo, cudaStream_t st);
int sgemm_tri(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A,
              int64_t lda, const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int tri,
              cudaStream_t st);

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

// The same ranking with 16 lanes per element, each lane counting every 16th
// key of a shared-memory copy of the whole diagonal (dynamic smem, 4d bytes),
// so d * 16 threads share the d^2 comparisons.
constexpr int RANK_LANES = 16;
__global__ void act_order_rank16_kernel(const float* __restrict__ h, int64_t d, int64_t ldh,
                                        int32_t* __restrict__ perm) {
  extern __shared__ float diag[];
  for (int64_t t = threadIdx.x; t < d; t += blockDim.x) diag[t] = h[t * ldh + t];
  __syncthreads();
  const int sub = threadIdx.x & (RANK_LANES - 1);
  const int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) / RANK_LANES;
  const float ki = (i < d) ? diag[i] : 0.f;
  int rank = 0;
#pragma unroll 4
  for (int64_t j = sub; j < d; j += RANK_LANES) {
    const float kj = diag[j];
    rank += key_gt(kj, ki) || (key_eq(kj, ki) && j > i);
  }
#pragma unroll
  for (int o = RANK_LANES / 2; o > 0; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
  if (i < d && sub == 0) perm[rank] = (int32_t)i;
}

__global__ void iota_kernel(int32_t* perm, int64_t d) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < d) perm[i] = (int32_t)i;
}

int act_order_perm(const float* h, int64_t d, int64_t ldh, int ordering, int32_t* perm,
                   cudaStream_t st) {
  if (d == 0) return GQ_OK;
  unsigned blocks = (unsigned)ceil_div(d, 256);
  const size_t diag_bytes = (size_t)d * sizeof(float);
  if (ordering == 0) {
    iota_kernel<<<blocks, 256, 0, st>>>(perm, d);
  } else if (diag_bytes <= 200 * 1024) {
    static int attr_device = -1;
    int dev = 0;
    GQ_CHECK_CUDA(cudaGetDevice(&dev));
    if (attr_device != dev) {
      GQ_CHECK_CUDA(cudaFuncSetAttribute(act_order_rank16_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      attr_device = dev;
    }
    act_order_rank16_kernel<<<(unsigned)ceil_div(d * RANK_LANES, 256), 256, diag_bytes, st>>>(
        h, d, ldh, perm);
  } else {
    act_order_rank_kernel<<<blocks, 256, 0, st>>>(h, d, ldh, perm);
  }
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

// Row i of the output is a gathered row of h: rows are read whole and
// coalesced into shared memory (n floats), then permuted out of it.
//   lower: ht[i][j] = h[q_i][q_j] + damp * mean * (i == j) for j <= i, 0 for
//          j > i, with q = the permutation reversed (q_i = p[n-1-i]);
//   full:  hd[i][j] = h[p_i][p_j] + damp * mean * (i == j).
template <bool LOWER>
__global__ void damp_permute_rows_kernel(const float* __restrict__ h, int64_t n, int64_t ldh,
                                         const int32_t* __restrict__ perm,
                                         const float* __restrict__ mean, float damp,
                                         float* __restrict__ out) {
  extern __shared__ float srow[];
  const float dv = damp * mean[0];
  for (int64_t i = blockIdx.x; i < n; i += gridDim.x) {
    const int64_t ri = LOWER ? (n - 1 - i) : i;
    const int64_t pi = perm ? perm[ri] : ri;
    __syncthreads();
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) srow[c] = h[pi * ldh + c];
    __syncthreads();
    for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
      float v = 0.f;
      if (!LOWER || j <= i) {
        const int64_t rj = LOWER ? (n - 1 - j) : j;
        v = srow[perm ? perm[rj] : rj];
        if (i == j) v = v + dv;
      }
      out[i * n + j] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Diagonal blocks of NB x NB are factored and inverted by one 512-thread CTA
// in shared memory, in four sub-panels of 32 columns (right-looking):
//   1. warp 0 factors the 32 x 32 diagonal sub-block with lane i holding row i
//      in registers (columns published by warp shuffles, no block barrier),
//      then inverts it with lane c solving L x = e_c;
//   2. all warps form the panel below, L21 = A21 X11^T (X11 = L11^-1);
//   3. all warps apply the rank-32 trailing update A22 -= L21 L21^T.
// The 128 x 128 inverse is then completed block row by block row,
// X_ij = -X_ii sum_k L_ik X_kj.  The block's inverse (not L) is written back:
// the panel solve below and the triangular inverse of the whole factor only
// need L^-1 on the diagonal.
constexpr int NB = 128;
constexpr int SUB = 32;
constexpr int DIAG_THREADS = 512;
constexpr int DIAG_WARPS = DIAG_THREADS / 32;
constexpr int DP = NB + 1;  // shared-memory pitch: row-strided lane reads hit distinct banks
constexpr size_t DIAG_SMEM = (size_t)(2 * NB + SUB) * DP * sizeof(float) + SUB * sizeof(float);

// acc[q][s] = sum_{k < K} A[r_q DP + k] * B(k, lane + 32s) for rows r_q = r0 + rstride * q
// below M and s < ns, where B(k, c) = B[c DP + k] (NT) or B[k DP + c] (NN).  Row reads
// are warp broadcasts; column reads are lane-contiguous (NN) or lane-strided by the odd
// pitch (NT).  Sums run over k in increasing order.
template <bool NT>
__device__ __forceinline__ void smem_mm(const float* A, const float* B, int M, int ns, int K,
                                        float (&acc)[6][3], int r0, int rstride) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < 6; ++q)
#pragma unroll
    for (int s = 0; s < 3; ++s) acc[q][s] = 0.f;
#pragma unroll 4
  for (int k = 0; k < K; ++k) {
    float b[3];
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      const int c = lane + 32 * s;
      b[s] = (s < ns) ? (NT ? B[c * DP + k] : B[k * DP + c]) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < 6; ++q) {
      const int r = r0 + rstride * q;
      if (r < M) {
        const float av = A[r * DP + k];
#pragma unroll
        for (int s = 0; s < 3; ++s) acc[q][s] = fmaf(av, b[s], acc[q][s]);
      }
    }
  }
}

// Warp-level Cholesky + inverse of the 32 x 32 sub-block at S[c0][c0]: L goes
// back to S, L^-1 to X.  rdiag: 32 floats of scratch.  Returns true (uniform)
// if a pivot was not > 0 or not finite; that pivot is replaced by 1.
__device__ bool sub_factor(float* S, float* X, float* rdiag, int c0) {
  const unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  float r[SUB];
#pragma unroll
  for (int k = 0; k < SUB; ++k) r[k] = S[(c0 + lane) * DP + c0 + k];
  bool bad = false;
  float my_rinv = 1.f;
#pragma unroll
  for (int j = 0; j < SUB; ++j) {
    float djj = __shfl_sync(FULL, r[j], j);
    if (!(djj > 0.f) || !isfinite(djj)) {
      bad = true;
      djj = 1.f;
    }
    // rsqrtf (2 ulp) keeps the serial pivot chain short; the factor's own
    // float32 rounding error is orders of magnitude larger
    const float rl = rsqrtf(djj);
    const float ljj = djj * rl;
    if (lane == j) my_rinv = rl;
    const float lij = (lane < j) ? 0.f : ((lane == j) ? ljj : r[j] * rl);
    r[j] = lij;
#pragma unroll
    for (int k = j + 1; k < SUB; ++k) r[k] = fmaf(-lij, __shfl_sync(FULL, lij, k), r[k]);
  }
#pragma unroll
  for (int k = 0; k < SUB; ++k) S[(c0 + lane) * DP + c0 + k] = r[k];
  rdiag[lane] = my_rinv;
  __syncwarp();
  // column `lane` of L^-1 by right-looking forward substitution: once x[k]
  // is final it is removed from every later row (L columns read as
  // broadcasts).  Each x[i] receives the same fmaf sequence as a dot product
  // over k < i would, but the dependent chain is one fmaf + one multiply per
  // column instead of the whole dot product.
  float x[SUB];
#pragma unroll
  for (int i = 0; i < SUB; ++i) x[i] = (i == lane) ? 1.f : 0.f;
#pragma unroll
  for (int k = 0; k < SUB; ++k) {
    x[k] = x[k] * rdiag[k];
#pragma unroll
    for (int i = k + 1; i < SUB; ++i) x[i] = fmaf(-S[(c0 + i) * DP + c0 + k], x[k], x[i]);
  }
#pragma unroll
  for (int i = 0; i < SUB; ++i) X[(c0 + i) * DP + c0 + lane] = x[i];
  return bad;
}

// Cholesky of the kb x kb lower block at a (ld lda); a receives L^-1 (strict
// upper part zeroed).  Rows/columns beyond kb are treated as identity.
__global__ void __launch_bounds__(DIAG_THREADS)
potrf_diag_kernel(float* __restrict__ a, int64_t lda, int kb, int* __restrict__ status) {
  extern __shared__ float smem[];
  float* S = smem;               // NB x DP: the block, becoming L
  float* X = S + NB * DP;        // NB x DP: L^-1
  float* W = X + NB * DP;        // SUB x DP: block-row products of the inverse
  float* rdiag = W + SUB * DP;   // SUB
  __shared__ int bad;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) bad = 0;
  // block -> shared memory with every global load of a thread in flight at once
  constexpr int PER_THREAD = NB * NB / DIAG_THREADS;  // 32
  if (kb == NB && (lda & 3) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0) {
    float4 v[PER_THREAD / 4];
#pragma unroll
    for (int it = 0; it < PER_THREAD / 4; ++it) {
      const int e4 = threadIdx.x + it * DIAG_THREADS;  // float4 index, 32 per row
      v[it] = *reinterpret_cast<const float4*>(a + (int64_t)(e4 >> 5) * lda + ((e4 & 31) << 2));
    }
#pragma unroll
    for (int it = 0; it < PER_THREAD / 4; ++it) {
      const int e4 = threadIdx.x + it * DIAG_THREADS;
      const int r = e4 >> 5, c = (e4 & 31) << 2;
      S[r * DP + c + 0] = (c + 0 <= r) ? v[it].x : 0.f;
      S[r * DP + c + 1] = (c + 1 <= r) ? v[it].y : 0.f;
      S[r * DP + c + 2] = (c + 2 <= r) ? v[it].z : 0.f;
      S[r * DP + c + 3] = (c + 3 <= r) ? v[it].w : 0.f;
    }
  } else {
    float v[PER_THREAD];
#pragma unroll
    for (int it = 0; it < PER_THREAD; ++it) {
      const int e = threadIdx.x + it * DIAG_THREADS, r = e / NB, c = e % NB;
      v[it] = (r < kb && c <= r) ? a[r * lda + c] : 0.f;
    }
#pragma unroll
    for (int it = 0; it < PER_THREAD; ++it) {
      const int e = threadIdx.x + it * DIAG_THREADS, r = e / NB, c = e % NB;
      S[r * DP + c] = (r < kb && c < kb) ? v[it] : ((r == c) ? 1.f : 0.f);
    }
  }
#pragma unroll 8
  for (int e = threadIdx.x; e < NB * NB; e += DIAG_THREADS) X[(e / NB) * DP + e % NB] = 0.f;
  __syncthreads();
  float acc[6][3];
  for (int c0 = 0; c0 < NB; c0 += SUB) {
    if (w == 0) {
      if (sub_factor(S, X, rdiag, c0) && lane == 0) bad = 1;
    }
    __syncthreads();
    const int m = NB - c0 - SUB;
    if (m == 0) break;
    float* panel = S + (c0 + SUB) * DP + c0;
    // L21 = A21 X11^T
    smem_mm<true>(panel, X + c0 * DP + c0, m, 1, SUB, acc, w, DIAG_WARPS);
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 6; ++q)
      if (w + DIAG_WARPS * q < m) panel[(w + DIAG_WARPS * q) * DP + lane] = acc[q][0];
    __syncthreads();
    // A22 -= L21 L21^T (lower part)
    smem_mm<true>(panel, panel, m, m / 32, SUB, acc, w, DIAG_WARPS);
    float* a22 = panel + SUB;
#pragma unroll
    for (int q = 0; q < 6; ++q)
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        const int r = w + DIAG_WARPS * q, c = lane + 32 * s;
        if (r < m && s < m / 32 && c <= r) a22[r * DP + c] -= acc[q][s];
      }
    __syncthreads();
  }
  // off-diagonal blocks of L^-1, block row by block row
  for (int i = 1; i < NB / SUB; ++i) {
    smem_mm<false>(S + SUB * i * DP, X, SUB, i, SUB * i, acc, w, DIAG_WARPS);  // W = L[i, :i] X[:i, :i]
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
      for (int s = 0; s < 3; ++s)
        if (s < i) W[(w + DIAG_WARPS * q) * DP + lane + 32 * s] = acc[q][s];
    __syncthreads();
    smem_mm<false>(X + SUB * i * DP + SUB * i, W, SUB, i, SUB, acc, w, DIAG_WARPS);  // -X_ii W
#pragma unroll
    for (int q = 0; q < 2; ++q)
#pragma unroll
      for (int s = 0; s < 3; ++s)
        if (s < i) X[(SUB * i + w + DIAG_WARPS * q) * DP + lane + 32 * s] = -acc[q][s];
    __syncthreads();
  }
  for (int e = threadIdx.x; e < NB * NB; e += DIAG_THREADS) {
    const int r = e / NB, c = e % NB;
    if (r < kb && c < kb) a[r * lda + c] = (c <= r) ? X[r * DP + c] : 0.f;
  }
  if (threadIdx.x == 0 && bad) atomicExch(status, GQ_DEVERR_NOTPD);
}

// u[i][j] = linv[n-1-i][n-1-j], one block per row (both sides coalesced)
__global__ void reverse_copy_kernel(const float* __restrict__ linv, int64_t n, int64_t ldl,
                                    float* __restrict__ u, int64_t ldu) {
  for (int64_t i = blockIdx.x; i < n; i += gridDim.x) {
    const float* src = linv + (n - 1 - i) * ldl + (n - 1);
    for (int64_t j = threadIdx.x; j < n; j += blockDim.x) u[i * ldu + j] = src[-j];
  }
}

int transpose2d(const float* src, int64_t rows, int64_t cols, int64_t lds, float* dst, int64_t ldd,
                cudaStream_t st);

// In-place inverse Cholesky of the n x n lower triangle of a (ld lda): on
// return the lower triangle holds X = L^-1, where A = L L^T.  The strict upper
// triangle must be zero on entry (the leaves keep their own diagonal blocks'
// upper parts zero).  Recursive on a split n = n1 + n2 (n1 a multiple of NB):
//   X11 = rec(A11);  L21 = A21 X11^T;  A22 -= L21 L21^T;  X22 = rec(A22);
//   X21 = -X22 L21 X11,
// i.e. Cholesky (n^3/3) and triangular inverse (n^3/3) interleaved, with the
// product operands' zero triangles skipped tile by tile.  Every GEMM has both
// operands K-major (tensor-core path): X11^T is formed by a transpose and the
// last product is taken as X21 = -X22 Tt^T with Tt = X11^T L21^T.
// scratch: n1 * n floats suffice (n1 <= n / 2 + NB).
constexpr int MAX_ROW_BYTES = 220 * 1024;  // the row-staged permute holds one row of h

int diag_kernel_setup() {
  static int attr_device = -1;
  int dev = 0;
  GQ_CHECK_CUDA(cudaGetDevice(&dev));
  if (attr_device != dev) {
    GQ_CHECK_CUDA(cudaFuncSetAttribute(potrf_diag_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)DIAG_SMEM));
    GQ_CHECK_CUDA(cudaFuncSetAttribute(damp_permute_rows_kernel<true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_ROW_BYTES));
    GQ_CHECK_CUDA(cudaFuncSetAttribute(damp_permute_rows_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_ROW_BYTES));
    attr_device = dev;
  }
  return GQ_OK;
}

int inv_chol_rec(float* a, int64_t n, int64_t lda, float* scratch, int* status, cudaStream_t st) {
  if (n <= NB) {
    potrf_diag_kernel<<<1, DIAG_THREADS, DIAG_SMEM, st>>>(a, lda, (int)n, status);
    return check_launch("potrf_diag");
  }
  int64_t n1 = ((n / 2 + NB - 1) / NB) * NB;
  if (n1 >= n) n1 = n - NB;
  const int64_t n2 = n - n1;
  float* a11 = a;
  float* a21 = a + n1 * lda;
  float* a22 = a21 + n1;
  GQ_TRY(inv_chol_rec(a11, n1, lda, scratch, status, st));
  float* l21 = scratch;  // n2 x n1
  GQ_TRY(sgemm_tri(0, 1, n2, n1, n1, 1.f, a21, lda, a11, lda, 0.f, l21, n1, 3, st));
  GQ_TRY(sgemm(0, 1, n2, n2, n1, -1.f, l21, n1, l21, n1, 1.f, a22, lda, 1, st));
  GQ_CHECK_CUDA(cudaMemcpy2DAsync(a21, lda * sizeof(float), l21, n1 * sizeof(float),
                                  n1 * sizeof(float), n2, cudaMemcpyDeviceToDevice, st));
  float* tt = scratch;            // n1 x n2: Tt = X11^T L21^T
  float* xt = scratch + n1 * n2;  // n1 x n1: X11^T
  GQ_TRY(transpose2d(a11, n1, n1, lda, xt, n1, st));
  GQ_TRY(sgemm_tri(0, 1, n1, n2, n1, 1.f, xt, n1, a21, lda, 0.f, tt, n2, 1, st));
  GQ_TRY(inv_chol_rec(a22, n2, lda, scratch + n1 * n2, status, st));
  GQ_TRY(sgemm_tri(0, 1, n2, n1, n2, -1.f, a22, lda, tt, n2, 0.f, a21, lda, 2, st));
  return GQ_OK;
}

int64_t hessian_ws_floats(int64_t d) {
  int64_t half = d / 2 + NB;
  return d * d + half * (d + NB) + 64;
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

int gq_hessian_factor_attempt(const float* h, int64_t d, int64_t ldh, const int32_t* perm,
                              double damp_percent, int attempt, float* u, int64_t ldu,
                              float* hd_out, void* workspace, int64_t workspace_bytes, int* status,
                              void* stream) {
  GQ_REQUIRE(h != nullptr && u != nullptr && status != nullptr,
             "gq_hessian_factor_attempt: NULL h, u or status");
  GQ_REQUIRE(d > 0 && ldh >= d && ldu >= d, "gq_hessian_factor_attempt: bad shape");
  GQ_REQUIRE(workspace_bytes >= gq_hessian_factor_workspace_size(d),
             "gq_hessian_factor_attempt: workspace too small (%lld < %lld)",
             (long long)workspace_bytes, (long long)gq_hessian_factor_workspace_size(d));
  GQ_REQUIRE(damp_percent >= 0.0, "gq_hessian_factor_attempt: negative damp_percent");
  GQ_REQUIRE(attempt >= 0 && attempt < 5, "gq_hessian_factor_attempt: attempt must be 0..4");
  GQ_REQUIRE(d * (int64_t)sizeof(float) <= gq::MAX_ROW_BYTES,
             "gq_hessian_factor_attempt: d = %lld exceeds %d", (long long)d,
             gq::MAX_ROW_BYTES / (int)sizeof(float));
  cudaStream_t st = gq::as_stream(stream);
  float* ws = reinterpret_cast<float*>(workspace);
  float* ht = ws;                                  // d*d
  float* scratch = ht + d * d;                     // (d/2+NB) x (d+NB)
  int64_t half = d / 2 + gq::NB;
  float* mean = scratch + half * (d + gq::NB);     // 1 float
  GQ_TRY(gq::diag_kernel_setup());
  gq::diag_mean_kernel<<<1, 1024, 0, st>>>(h, d, ldh, mean);
  GQ_TRY(gq::check_launch("diag_mean"));
  const double damp = std::pow(10.0, attempt) * damp_percent;
  GQ_CHECK_CUDA(cudaMemsetAsync(status, 0, sizeof(int), st));
  const unsigned rows_grid = (unsigned)std::min<int64_t>(d, 148 * 16);
  const size_t row_bytes = (size_t)d * sizeof(float);
  gq::damp_permute_rows_kernel<true><<<rows_grid, 256, row_bytes, st>>>(h, d, ldh, perm, mean,
                                                                        (float)damp, ht);
  GQ_TRY(gq::check_launch("damp_permute"));
  if (hd_out) {
    gq::damp_permute_rows_kernel<false><<<rows_grid, 256, row_bytes, st>>>(h, d, ldh, perm, mean,
                                                                           (float)damp, hd_out);
    GQ_TRY(gq::check_launch("damp_permute"));
  }
  // L^-1 in place (lower triangle; the strict upper part is zero), then U = J L^-1 J
  GQ_TRY(gq::inv_chol_rec(ht, d, d, scratch, status, st));
  gq::reverse_copy_kernel<<<rows_grid, 256, 0, st>>>(ht, d, d, u, ldu);
  return gq::check_launch("reverse_copy");
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
  int64_t half = d / 2 + gq::NB;
  float* mean = ws + d * d + half * (d + gq::NB);  // 1 float
  int* status = reinterpret_cast<int*>(mean + 16);  // 1 int
  for (int attempt = 0; attempt < 5; ++attempt) {
    GQ_TRY(gq_hessian_factor_attempt(h, d, ldh, perm, damp_percent, attempt, u, ldu, hd_out,
                                     workspace, workspace_bytes, status, stream));
    int host_status = 0;
    GQ_CHECK_CUDA(cudaMemcpyAsync(&host_status, status, sizeof(int), cudaMemcpyDeviceToHost, st));
    GQ_CHECK_CUDA(cudaStreamSynchronize(st));
    if (host_status != gq::GQ_DEVERR_NONE) continue;
    if (attempt_out) *attempt_out = attempt;
    return GQ_OK;
  }
  if (attempt_out) *attempt_out = -1;
  return gq::fail(GQ_ENOTPD, "gq_hessian_factor: damped Hessian not positive definite after 5 attempts");
}

}  // extern "C"
