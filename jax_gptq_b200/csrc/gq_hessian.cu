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
#include <map>
#include <mutex>
#include <utility>

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
// in shared memory: four 32-column sub-panels, right-looking, with the
// block's inverse completed along the way, X_ij = -X_ii sum_k L_ik X_kj.
// Only the inverse is written back: the panel solve of the recursion and the
// triangular inverse of the whole factor need L^-1 on the diagonal, not L.
//
// The 32 pivots of a sub-panel form the serial chain.  Warp 0 factors and
// inverts each 32 x 32 diagonal sub-block in registers (lane i holds row i;
// columns published through shared memory) while the 12 warps that do not
// share its scheduler do every piece of the parallel work that does not feed
// the next pivot (look-ahead):
//   phase p, warp 0:     sub-block p -> X_pp
//   phase p, 12 warps:   the trailing update from panel p-1 outside block
//                        column p, W_pj = sum_{k<p} L_pk X_kj, and the global
//                        stores of finished rows of the inverse;
//   then all 16 warps:   the panel L_ip = A_ip X_pp^T, X_pj = -X_pp W_pj, and
//                        the update of the next diagonal sub-block.
// Every product sums over k in increasing order from zero with fmaf and each
// block receives the updates of panels 0, 1, ... in order, so the result does
// not depend on how the work is split between warps.
constexpr int NB = 128;
constexpr int SUB = 32;
constexpr int DIAG_THREADS = 512;
constexpr int DIAG_WARPS = DIAG_THREADS / 32;
constexpr int DP = NB + 1;   // shared-memory pitch: row-strided lane reads hit distinct banks
constexpr int LTP = SUB + 4;  // pitch of the transposed sub-block (rows 16-byte aligned)
constexpr size_t DIAG_SMEM = ((size_t)(2 * NB + SUB) * DP + (size_t)SUB * LTP + 3 * SUB) * sizeof(float);

// acc[q][s] = sum_{k0 <= k < k1} A(r_q, k) B(k, c_s) for the rows r_q = w + nw q
// (q < QN, r_q < nrows) and columns c_s = lane + 32 s, with A(r, k) = A[r DP + k]
// and B(k, c) = B[c DP + k] (NT) or B[k DP + c] (NN).  Row reads are warp
// broadcasts; column reads are lane-contiguous (NN) or lane-strided by the odd
// pitch (NT), so no access has a bank conflict.
template <bool NT, int QN, int NS>
__device__ __forceinline__ void bprod(const float* __restrict__ A, const float* __restrict__ B,
                                      int nrows, int w, int nw, int k0, int k1,
                                      float (&acc)[QN][NS]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < QN; ++q)
#pragma unroll
    for (int s = 0; s < NS; ++s) acc[q][s] = 0.f;
#pragma unroll 4
  for (int k = k0; k < k1; ++k) {
    float b[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const int c = lane + 32 * s;
      b[s] = NT ? B[c * DP + k] : B[k * DP + c];
    }
#pragma unroll
    for (int q = 0; q < QN; ++q) {
      const int r = w + nw * q;
      if (r < nrows) {
        const float av = A[r * DP + k];
#pragma unroll
        for (int s = 0; s < NS; ++s) acc[q][s] = fmaf(av, b[s], acc[q][s]);
      }
    }
  }
}

// Warp-level Cholesky + inverse of a 32 x 32 block held as r (lane i: row i,
// lower part; the upper part is ignored).  L^-1 goes to xd (pitch DP, zeros
// above the diagonal).  Scratch (16-byte aligned): lt, 32 x LTP floats; cb,
// 2 x 32 floats; rdiag, 32 floats.
// Column j of the trailing matrix is published in cb as soon as it is final
// (one pivot ahead) and read back as float4 broadcasts, so each lane forms
// the whole column of L itself, l_kj = a_kj / l_jj, and takes the pivot from
// it; the read-back of the next column is issued before the current pivot's
// bulk updates, which hide its latency.
// Returns true (uniform) if a pivot was not > 0 or not finite; that pivot is
// replaced by 1.
__device__ bool sub_factor(float (&r)[SUB], float* xd, float* lt, float* cb, float* rdiag) {
  const int lane = threadIdx.x & 31;
  cb[lane] = r[0];
  __syncwarp();
  // column j of the trailing block, published one pivot ahead; the pivot is
  // its entry j (lane j's own r[j], which every lane reads here)
  float cv[SUB];
  {
    const float4* c4 = reinterpret_cast<const float4*>(cb);
#pragma unroll
    for (int g = 0; g < SUB / 4; ++g) {
      const float4 v = c4[g];
      cv[4 * g + 0] = v.x;
      cv[4 * g + 1] = v.y;
      cv[4 * g + 2] = v.z;
      cv[4 * g + 3] = v.w;
    }
  }
  bool bad = false;
#pragma unroll
  for (int j = 0; j < SUB; ++j) {
    float djj = cv[j];
    if (!(djj > 0.f) || !isfinite(djj)) {
      bad = true;
      djj = 1.f;
    }
    // rsqrtf (2 ulp) keeps the serial pivot chain short; the factor's own
    // float32 rounding error is orders of magnitude larger
    const float rl = rsqrtf(djj);
    if (lane == 0) rdiag[j] = rl;
    const float lij = (lane < j) ? 0.f : ((lane == j) ? djj * rl : r[j] * rl);
    r[j] = lij;
    if (j + 1 < SUB) {
      // the next column first: update, publish, and start reading it back so
      // the load overlaps this pivot's remaining updates
      r[j + 1] = fmaf(-lij, cv[j + 1] * rl, r[j + 1]);
      // double-buffered: this buffer's previous readers are past the last __syncwarp
      cb[((j + 1) & 1) * SUB + lane] = r[j + 1];
      __syncwarp();
      float nx[SUB];
      const float4* c4 = reinterpret_cast<const float4*>(cb + ((j + 1) & 1) * SUB);
#pragma unroll
      for (int g = (j + 1) / 4; g < SUB / 4; ++g) {
        const float4 v = c4[g];
        nx[4 * g + 0] = v.x;
        nx[4 * g + 1] = v.y;
        nx[4 * g + 2] = v.z;
        nx[4 * g + 3] = v.w;
      }
      // off the pivot chain: l_ij l_kj = (l_ij rl) a_kj, one FMA per entry
      const float lr = lij * rl;
#pragma unroll
      for (int k = j + 2; k < SUB; ++k) r[k] = fmaf(-lr, cv[k], r[k]);
#pragma unroll
      for (int k = j + 1; k < SUB; ++k) cv[k] = nx[k];
    }
  }
  // L transposed, so that a column of L is one run of float4 broadcasts
#pragma unroll
  for (int k = 0; k < SUB; ++k) lt[k * LTP + lane] = r[k];
  __syncwarp();
  // column `lane` of L^-1 by right-looking forward substitution: once x[k] is
  // final it is removed from every later row
  float x[SUB];
#pragma unroll
  for (int i = 0; i < SUB; ++i) x[i] = (i == lane) ? 1.f : 0.f;
#pragma unroll
  for (int k = 0; k < SUB; ++k) {
    x[k] = x[k] * rdiag[k];
    const float4* col = reinterpret_cast<const float4*>(lt + k * LTP);
#pragma unroll
    for (int g = (k + 1) / 4; g < SUB / 4; ++g) {
      const float4 l4 = col[g];
      const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * g + e;
        if (i > k) x[i] = fmaf(-lv[e], x[k], x[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < SUB; ++i) xd[i * DP + lane] = x[i];
  __syncwarp();
  return bad;
}

// Rows [32 rb, 32 rb + 32) of the block's inverse to global memory (zeros
// above the diagonal), by threads t0 .. t0 + nt - 1.
__device__ __forceinline__ void store_inverse_rows(float* __restrict__ a, int64_t lda, int kb,
                                                   bool vec, const float* X, int rb, int t,
                                                   int nt) {
  if (vec) {
    for (int e4 = t; e4 < SUB * NB / 4; e4 += nt) {
      const int r = SUB * rb + (e4 >> 5), c = (e4 & 31) << 2;
      float4 v;
      v.x = (c + 0 <= r) ? X[r * DP + c + 0] : 0.f;
      v.y = (c + 1 <= r) ? X[r * DP + c + 1] : 0.f;
      v.z = (c + 2 <= r) ? X[r * DP + c + 2] : 0.f;
      v.w = (c + 3 <= r) ? X[r * DP + c + 3] : 0.f;
      *reinterpret_cast<float4*>(a + (int64_t)r * lda + c) = v;
    }
  } else {
    for (int e = t; e < SUB * NB; e += nt) {
      const int r = SUB * rb + e / NB, c = e % NB;
      if (r < kb && c < kb) a[(int64_t)r * lda + c] = (c <= r) ? X[r * DP + c] : 0.f;
    }
  }
}

// Cholesky of the kb x kb lower block at a (ld lda); a receives L^-1 (strict
// upper part zeroed).  Rows/columns beyond kb are treated as identity.
__global__ void __launch_bounds__(DIAG_THREADS)
potrf_diag_kernel(float* __restrict__ a, int64_t lda, int kb, int* __restrict__ status) {
  extern __shared__ __align__(16) float smem[];
  float* S = smem;               // NB x DP: the block; off-diagonal blocks become L
  float* X = S + NB * DP;        // NB x DP: L^-1 (blocks above the diagonal never written)
  float* Wb = X + NB * DP;       // SUB x DP: W_pj = sum_k L_pk X_kj of the current block row
  float* lt = Wb + SUB * DP;     // SUB x LTP: warp 0's transposed sub-block
  float* cb = lt + SUB * LTP;    // 2 x SUB: warp 0's published pivot columns
  float* rdiag = cb + 2 * SUB;   // SUB: reciprocal pivots
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool vec = kb == NB && (lda & 3) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0;
  // look-ahead warps: every warp not on warp 0's scheduler (warps 4, 8, 12
  // share it), so the pivot chain is never waiting for an issue slot
  const bool la = (w & 3) != 0;
  const int lw = w - 1 - (w >> 2);
  constexpr int LW = DIAG_WARPS - DIAG_WARPS / 4;
  const int lt_thread = lw * 32 + lane;
  constexpr int LT_THREADS = 32 * LW;
  const int ld_thread = threadIdx.x - 32;  // warps 1-15 load rows 32..127
  constexpr int LD_THREADS = DIAG_THREADS - 32;
  bool bad = false;  // warp 0 only
  float r[SUB];
  float acc6[6][1], acc6c[6][3], acc3[3][2], acc2[2][1], acc2b[2][2], acc2c[2][3], acc3b[3][1];

  // ---- phase 0: warp 0 loads and factors sub-block 0 while warps 1-15 load rows 32..127
  if (w == 0) {
    if (vec) {
#pragma unroll
      for (int g = 0; g < SUB / 4; ++g) {
        const float4 v = *reinterpret_cast<const float4*>(a + (int64_t)lane * lda + 4 * g);
        r[4 * g + 0] = (4 * g + 0 <= lane) ? v.x : 0.f;
        r[4 * g + 1] = (4 * g + 1 <= lane) ? v.y : 0.f;
        r[4 * g + 2] = (4 * g + 2 <= lane) ? v.z : 0.f;
        r[4 * g + 3] = (4 * g + 3 <= lane) ? v.w : 0.f;
      }
    } else {
#pragma unroll
      for (int k = 0; k < SUB; ++k)
        r[k] = (lane < kb && k < kb) ? ((k <= lane) ? a[(int64_t)lane * lda + k] : 0.f)
                                     : ((lane == k) ? 1.f : 0.f);
    }
    bad |= sub_factor(r, X, lt, cb, rdiag);
  } else if (vec) {
    constexpr int N4 = (NB - SUB) * NB / 4;  // float4s in rows 32..127
    constexpr int IT = (N4 + LD_THREADS - 1) / LD_THREADS;
    float4 v[IT];
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int e4 = ld_thread + it * LD_THREADS;
      if (e4 < N4)
        v[it] = *reinterpret_cast<const float4*>(a + (int64_t)(SUB + (e4 >> 5)) * lda +
                                                 ((e4 & 31) << 2));
    }
#pragma unroll
    for (int it = 0; it < IT; ++it) {
      const int e4 = ld_thread + it * LD_THREADS;
      if (e4 < N4) {
        const int rr = SUB + (e4 >> 5), c = (e4 & 31) << 2;
        S[rr * DP + c + 0] = (c + 0 <= rr) ? v[it].x : 0.f;
        S[rr * DP + c + 1] = (c + 1 <= rr) ? v[it].y : 0.f;
        S[rr * DP + c + 2] = (c + 2 <= rr) ? v[it].z : 0.f;
        S[rr * DP + c + 3] = (c + 3 <= rr) ? v[it].w : 0.f;
      }
    }
  } else {
    for (int e = ld_thread; e < (NB - SUB) * NB; e += LD_THREADS) {
      const int rr = SUB + e / NB, c = e % NB;
      const float v = (rr < kb && c <= rr) ? a[(int64_t)rr * lda + c] : 0.f;
      S[rr * DP + c] = (rr < kb && c < kb) ? v : ((rr == c) ? 1.f : 0.f);
    }
  }
  __syncthreads();
  // panel 0: L_i0 = A_i0 X_00^T (rows 32..127)
  bprod<true, 6, 1>(S + SUB * DP, X, NB - SUB, w, DIAG_WARPS, 0, SUB, acc6);
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 6; ++q) {
    const int rr = w + DIAG_WARPS * q;
    if (rr < NB - SUB) S[(SUB + rr) * DP + lane] = acc6[q][0];
  }
  __syncthreads();
  // A_11 -= L_10 L_10^T
  bprod<true, 2, 1>(S + SUB * DP, S + SUB * DP, SUB, w, DIAG_WARPS, 0, SUB, acc2);
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int rr = w + DIAG_WARPS * q;
    if (lane <= rr) S[(SUB + rr) * DP + SUB + lane] -= acc2[q][0];
  }
  __syncthreads();

  // ---- phase 1
  if (w == 0) {
#pragma unroll
    for (int k = 0; k < SUB; ++k) r[k] = S[(SUB + lane) * DP + SUB + k];
    bad |= sub_factor(r, X + SUB * DP + SUB, lt, cb, rdiag);
  } else if (la) {
    // rows 64..127, columns 32..127: A -= L_i0 L_j0^T (lower part)
    bprod<true, 6, 3>(S + 2 * SUB * DP, S + SUB * DP, 2 * SUB, lw, LW, 0, SUB, acc6c);
#pragma unroll
    for (int q = 0; q < 6; ++q)
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        const int rr = lw + LW * q, c = lane + 32 * s;
        if (rr < 2 * SUB && SUB + c <= 2 * SUB + rr) S[(2 * SUB + rr) * DP + SUB + c] -= acc6c[q][s];
      }
    // W_10 = L_10 X_00
    bprod<false, 3, 1>(S + SUB * DP, X, SUB, lw, LW, 0, SUB, acc3b);
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const int rr = lw + LW * q;
      if (rr < SUB) Wb[rr * DP + lane] = acc3b[q][0];
    }
  }
  __syncthreads();
  // panel 1: L_i1 = A_i1 X_11^T (rows 64..127); X_10 = -X_11 W_10
  {
    float acc4[4][1];
    bprod<true, 4, 1>(S + 2 * SUB * DP, X + SUB * DP, 2 * SUB, w, DIAG_WARPS, SUB, 2 * SUB, acc4);
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int rr = w + DIAG_WARPS * q;
      if (rr < 2 * SUB) S[(2 * SUB + rr) * DP + SUB + lane] = acc4[q][0];
    }
  }
  bprod<false, 2, 1>(X + SUB * DP + SUB, Wb, SUB, w, DIAG_WARPS, 0, SUB, acc2);
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int rr = w + DIAG_WARPS * q;
    X[(SUB + rr) * DP + lane] = -acc2[q][0];
  }
  __syncthreads();
  // A_22 -= L_21 L_21^T
  bprod<true, 2, 1>(S + 2 * SUB * DP, S + 2 * SUB * DP, SUB, w, DIAG_WARPS, SUB, 2 * SUB, acc2);
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int rr = w + DIAG_WARPS * q;
    if (lane <= rr) S[(2 * SUB + rr) * DP + 2 * SUB + lane] -= acc2[q][0];
  }
  __syncthreads();

  // ---- phase 2
  if (w == 0) {
#pragma unroll
    for (int k = 0; k < SUB; ++k) r[k] = S[(2 * SUB + lane) * DP + 2 * SUB + k];
    bad |= sub_factor(r, X + 2 * SUB * DP + 2 * SUB, lt, cb, rdiag);
  } else if (la) {
    // rows 96..127, columns 64..127: A -= L_i1 L_j1^T (lower part)
    bprod<true, 3, 2>(S + 3 * SUB * DP, S + 2 * SUB * DP, SUB, lw, LW, SUB, 2 * SUB, acc3);
#pragma unroll
    for (int q = 0; q < 3; ++q)
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int rr = lw + LW * q, c = lane + 32 * s;
        if (rr < SUB && c <= SUB + rr) S[(3 * SUB + rr) * DP + 2 * SUB + c] -= acc3[q][s];
      }
    // W_20 = L_20 X_00 + L_21 X_10, W_21 = L_21 X_11
    bprod<false, 3, 1>(S + 2 * SUB * DP, X, SUB, lw, LW, 0, 2 * SUB, acc3b);
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const int rr = lw + LW * q;
      if (rr < SUB) Wb[rr * DP + lane] = acc3b[q][0];
    }
    bprod<false, 3, 1>(S + 2 * SUB * DP, X + SUB, SUB, lw, LW, SUB, 2 * SUB, acc3b);
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const int rr = lw + LW * q;
      if (rr < SUB) Wb[rr * DP + SUB + lane] = acc3b[q][0];
    }
    // rows 0..63 of the inverse are final
    store_inverse_rows(a, lda, kb, vec, X, 0, lt_thread, LT_THREADS);
    store_inverse_rows(a, lda, kb, vec, X, 1, lt_thread, LT_THREADS);
  }
  __syncthreads();
  // panel 2: L_32 = A_32 X_22^T; X_2j = -X_22 W_2j (j = 0, 1)
  bprod<true, 2, 1>(S + 3 * SUB * DP, X + 2 * SUB * DP, SUB, w, DIAG_WARPS, 2 * SUB, 3 * SUB, acc2);
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int rr = w + DIAG_WARPS * q;
    S[(3 * SUB + rr) * DP + 2 * SUB + lane] = acc2[q][0];
  }
  bprod<false, 2, 2>(X + 2 * SUB * DP + 2 * SUB, Wb, SUB, w, DIAG_WARPS, 0, SUB, acc2b);
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int rr = w + DIAG_WARPS * q;
      X[(2 * SUB + rr) * DP + lane + 32 * s] = -acc2b[q][s];
    }
  __syncthreads();
  // A_33 -= L_32 L_32^T
  bprod<true, 2, 1>(S + 3 * SUB * DP, S + 3 * SUB * DP, SUB, w, DIAG_WARPS, 2 * SUB, 3 * SUB, acc2);
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int rr = w + DIAG_WARPS * q;
    if (lane <= rr) S[(3 * SUB + rr) * DP + 3 * SUB + lane] -= acc2[q][0];
  }
  __syncthreads();

  // ---- phase 3
  if (w == 0) {
#pragma unroll
    for (int k = 0; k < SUB; ++k) r[k] = S[(3 * SUB + lane) * DP + 3 * SUB + k];
    bad |= sub_factor(r, X + 3 * SUB * DP + 3 * SUB, lt, cb, rdiag);
  } else if (la) {
    // W_3j = sum_{j <= k < 3} L_3k X_kj
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      bprod<false, 3, 1>(S + 3 * SUB * DP, X + SUB * j, SUB, lw, LW, SUB * j, 3 * SUB, acc3b);
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int rr = lw + LW * q;
        if (rr < SUB) Wb[rr * DP + SUB * j + lane] = acc3b[q][0];
      }
    }
    store_inverse_rows(a, lda, kb, vec, X, 2, lt_thread, LT_THREADS);
  }
  __syncthreads();
  // X_3j = -X_33 W_3j (j = 0, 1, 2)
  bprod<false, 2, 3>(X + 3 * SUB * DP + 3 * SUB, Wb, SUB, w, DIAG_WARPS, 0, SUB, acc2c);
#pragma unroll
  for (int q = 0; q < 2; ++q)
#pragma unroll
    for (int s = 0; s < 3; ++s) {
      const int rr = w + DIAG_WARPS * q;
      X[(3 * SUB + rr) * DP + lane + 32 * s] = -acc2c[q][s];
    }
  __syncthreads();
  store_inverse_rows(a, lda, kb, vec, X, 3, threadIdx.x, DIAG_THREADS);
  if (w == 0 && lane == 0 && bad) atomicExch(status, GQ_DEVERR_NOTPD);
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
//
// Tt depends only on X11 and L21, so it is formed on a side stream (same
// priority as the caller's) while the caller's stream runs the Schur update
// and rec(A22); the last product waits for it.  The critical path per split
// is then L21, the update, rec(A22) and X21.  All splits share the one side
// stream: each split's Tt is queued behind those of the splits that forked
// before it, which are smaller or finished long before it is needed, and a
// single extra stream per caller keeps the streams of a concurrent layer set
// within the device's hardware work queues (streams that share a queue wait
// on one another's pending dependencies).
//
// Scratch per split, in this order: L21 (n2 x n1), Tt (n1 x n2), X11^T
// (n1 x n1), then rec(A22)'s scratch; rec(A11) runs before any of them is
// written and reuses the same base.  inv_chol_scratch_floats(n) is the total.
constexpr int MAX_FORK_DEPTH = 24;

int64_t split_n1(int64_t n) {
  int64_t n1 = ((n / 2 + NB - 1) / NB) * NB;
  if (n1 >= n) n1 = n - NB;
  return n1;
}

int64_t inv_chol_scratch_floats(int64_t n) {
  if (n <= NB) return 0;
  const int64_t n1 = split_n1(n), n2 = n - n1;
  return std::max(inv_chol_scratch_floats(n1),
                  2 * n1 * n2 + n1 * n1 + inv_chol_scratch_floats(n2));
}

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

// The side stream and events of the recursion's forks, one set per (device,
// caller stream), created on first use with the caller stream's priority and
// kept for the life of the process.  Calls that share a caller stream must
// not run concurrently on different host threads (as for any stream).
struct Forks {
  cudaStream_t side;
  cudaEvent_t fork[MAX_FORK_DEPTH];
  cudaEvent_t join[MAX_FORK_DEPTH];
  // gq_factor_from_x_attempt: A11 formed, all of H formed (statistics stream)
  cudaEvent_t a11_ready, h_ready;
};

int forks_for(cudaStream_t st, Forks** out) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, Forks*> table;
  int dev = 0;
  GQ_CHECK_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  auto it = table.find({dev, st});
  if (it != table.end()) {
    *out = it->second;
    return GQ_OK;
  }
  int prio = 0;
  GQ_CHECK_CUDA(cudaStreamGetPriority(st, &prio));
  Forks* f = new Forks();
  GQ_CHECK_CUDA(cudaStreamCreateWithPriority(&f->side, cudaStreamNonBlocking, prio));
  for (int i = 0; i < MAX_FORK_DEPTH; ++i) {
    GQ_CHECK_CUDA(cudaEventCreateWithFlags(&f->fork[i], cudaEventDisableTiming));
    GQ_CHECK_CUDA(cudaEventCreateWithFlags(&f->join[i], cudaEventDisableTiming));
  }
  GQ_CHECK_CUDA(cudaEventCreateWithFlags(&f->a11_ready, cudaEventDisableTiming));
  GQ_CHECK_CUDA(cudaEventCreateWithFlags(&f->h_ready, cudaEventDisableTiming));
  table[{dev, st}] = f;
  *out = f;
  return GQ_OK;
}

int inv_chol_after_a11(float* a, int64_t n, int64_t lda, float* scratch, int* status,
                       cudaStream_t st, Forks* forks, int depth);

int inv_chol_rec(float* a, int64_t n, int64_t lda, float* scratch, int* status, cudaStream_t st,
                 Forks* forks, int depth) {
  if (n <= NB) {
    potrf_diag_kernel<<<1, DIAG_THREADS, DIAG_SMEM, st>>>(a, lda, (int)n, status);
    return check_launch("potrf_diag");
  }
  GQ_REQUIRE(depth < MAX_FORK_DEPTH, "inv_chol_rec: recursion deeper than %d", MAX_FORK_DEPTH);
  GQ_TRY(inv_chol_rec(a, split_n1(n), lda, scratch, status, st, forks, depth + 1));
  return inv_chol_after_a11(a, n, lda, scratch, status, st, forks, depth);
}

// The split's work after rec(A11): L21, the Schur update, rec(A22) and X21
// (Tt on the side stream).
int inv_chol_after_a11(float* a, int64_t n, int64_t lda, float* scratch, int* status,
                       cudaStream_t st, Forks* forks, int depth) {
  const int64_t n1 = split_n1(n), n2 = n - n1;
  float* a11 = a;
  float* a21 = a + n1 * lda;
  float* a22 = a21 + n1;
  float* l21 = scratch;            // n2 x n1
  float* tt = l21 + n2 * n1;       // n1 x n2: Tt = X11^T L21^T
  float* xt = tt + n1 * n2;        // n1 x n1: X11^T
  float* rest = xt + n1 * n1;      // rec(A22)'s scratch
  GQ_TRY(sgemm_tri(0, 1, n2, n1, n1, 1.f, a21, lda, a11, lda, 0.f, l21, n1, 3, st));
  cudaStream_t side = forks->side;
  GQ_CHECK_CUDA(cudaEventRecord(forks->fork[depth], st));
  GQ_CHECK_CUDA(cudaStreamWaitEvent(side, forks->fork[depth], 0));
  GQ_TRY(transpose2d(a11, n1, n1, lda, xt, n1, side));
  GQ_TRY(sgemm_tri(0, 1, n1, n2, n1, 1.f, xt, n1, l21, n1, 0.f, tt, n2, 1, side));
  GQ_CHECK_CUDA(cudaEventRecord(forks->join[depth], side));
  GQ_TRY(sgemm(0, 1, n2, n2, n1, -1.f, l21, n1, l21, n1, 1.f, a22, lda, 1, st));
  GQ_TRY(inv_chol_rec(a22, n2, lda, rest, status, st, forks, depth + 1));
  GQ_CHECK_CUDA(cudaStreamWaitEvent(st, forks->join[depth], 0));
  GQ_TRY(sgemm_tri(0, 1, n2, n1, n2, -1.f, a22, lda, tt, n2, 0.f, a21, lda, 2, st));
  return GQ_OK;
}

int inv_chol(float* a, int64_t n, int64_t lda, float* scratch, int* status, cudaStream_t st) {
  Forks* forks = nullptr;
  if (n > NB) GQ_TRY(forks_for(st, &forks));
  return inv_chol_rec(a, n, lda, scratch, status, st, forks, 0);
}

// Workspace: the damped, permuted copy (d x d), then the recursion's scratch
// from a 256-byte boundary, then the damping mean and the status word.
int64_t hessian_scratch_offset(int64_t d) { return (d * d + 63) / 64 * 64; }

int64_t hessian_ws_floats(int64_t d) {
  return hessian_scratch_offset(d) + inv_chol_scratch_floats(d) + 64;
}


// ---------------------------------------------------------------------------
// Factor straight from the activations (gq_factor_from_x_attempt).
//
// The factor's first split only needs the leading block A11 of the damped,
// permuted, reversed Hessian.  Its features are known once the diagonal of H
// is (act order sorts it), so the columns of X are gathered into that order
// and H is formed block by block: A11 first, then A21 and A22 while rec(A11)
// already runs on the chain stream.  Every element equals the one the
// one-shot path computes (the same tensor-core tile arithmetic on the same
// token order; a product and its mirror are the same bf16 x bf16 products),
// and the diagonal, the mean and the permutation come from the diagonal tiles
// of the original-order H, so u and perm are bit-identical to
// gq_syrk_bf16 -> gq_act_order_perm -> gq_hessian_factor_attempt.

// xr[t][i] = x[t][perm[d - 1 - i]] (bf16 bits); d % 8 == 0, rows 16-byte aligned.
__global__ void gather_cols_reversed_kernel(const uint16_t* __restrict__ x, int64_t tokens,
                                            int64_t d, int64_t ldx,
                                            const int32_t* __restrict__ perm,
                                            uint16_t* __restrict__ xr) {
  extern __shared__ __align__(16) uint8_t gsm[];
  int32_t* q = reinterpret_cast<int32_t*>(gsm);
  uint16_t* row = reinterpret_cast<uint16_t*>(gsm + ((d * 4 + 15) / 16) * 16);
  for (int64_t i = threadIdx.x; i < d; i += blockDim.x) q[i] = perm[d - 1 - i];
  for (int64_t t = blockIdx.x; t < tokens; t += gridDim.x) {
    __syncthreads();
    const uint16_t* src = x + t * ldx;
    for (int64_t c = (int64_t)threadIdx.x * 8; c < d; c += (int64_t)blockDim.x * 8)
      *reinterpret_cast<uint4*>(row + c) = *reinterpret_cast<const uint4*>(src + c);
    __syncthreads();
    uint16_t* dst = xr + t * d;
    for (int64_t i = (int64_t)threadIdx.x * 8; i < d; i += (int64_t)blockDim.x * 8) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        w[e] = (uint32_t)row[q[i + 2 * e]] | ((uint32_t)row[q[i + 2 * e + 1]] << 16);
      *reinterpret_cast<uint4*>(dst + i) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Diagonal block a[0:n, 0:n] (ld lda) whose upper triangle holds H: the lower
// triangle receives the mirror, the diagonal + damp * mean, the strict upper
// triangle zeros -- what damp_permute_rows_kernel<true> writes.  Block (bi, bj)
// with bj <= bi owns the 32 x 32 tiles (bi, bj) and (bj, bi).
__global__ void lower_damped_from_upper_kernel(float* __restrict__ a, int64_t n, int64_t lda,
                                               const float* __restrict__ mean, float damp) {
  __shared__ float tile[32][33];
  const int64_t bi = blockIdx.y, bj = blockIdx.x;
  if (bj > bi) return;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  const float dv = damp * mean[0];
  for (int r = ty; r < 32; r += 8) {  // upper tile (bj, bi)
    const int64_t i = bj * 32 + r, j = bi * 32 + tx;
    tile[r][tx] = (i < n && j < n) ? a[i * lda + j] : 0.f;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const int64_t i = bi * 32 + r, j = bj * 32 + tx;  // (i, j) in tile (bi, bj)
    if (i < n && j < n) {
      float v = 0.f;
      if (j < i) v = tile[tx][r];            // mirror of (j, i)
      else if (j == i) v = tile[r][tx] + dv;  // (bi == bj here)
      a[i * lda + j] = v;
    }
    if (bi > bj) {  // the upper tile's element (bj*32 + r, bi*32 + tx) -> 0
      const int64_t ui = bj * 32 + r, uj = bi * 32 + tx;
      if (ui < n && uj < n) a[ui * lda + uj] = 0.f;
    }
  }
}

namespace tc {
int launch(const void* xa, int64_t lda, const void* xb, int64_t ldb, int64_t K, int64_t M,
           int64_t N, float* c, int64_t ldc, int accumulate, int symmetric, cudaStream_t st,
           int diag_only);
}

int lower_damped_from_upper(float* a, int64_t n, int64_t lda, const float* mean, float damp,
                            cudaStream_t st) {
  if (n == 0) return GQ_OK;
  const int64_t nt = ceil_div(n, 32);
  lower_damped_from_upper_kernel<<<dim3((unsigned)nt, (unsigned)nt), dim3(32, 8), 0, st>>>(
      a, n, lda, mean, damp);
  return check_launch("lower_damped_from_upper");
}

// Workspace of the from-activations factor: the hessian factor's layout
// (working matrix, recursion scratch, mean), then the gathered activations.
int64_t factor_x_gather_offset(int64_t d) { return (hessian_ws_floats(d) * 4 + 255) / 256 * 256; }

}  // namespace gq

extern "C" {

int gq_act_order_perm(const float* h, int64_t d, int64_t ldh, int ordering, int32_t* perm,
                      void* stream) {
  GQ_REQUIRE(d >= 0 && ldh >= d, "gq_act_order_perm: bad shape");
  GQ_REQUIRE(ordering == 0 || ordering == 1, "gq_act_order_perm: ordering must be 0 or 1");
  GQ_REQUIRE(d < (1ll << 31), "gq_act_order_perm: d too large");
  return gq::act_order_perm(h, d, ldh, ordering, perm, gq::as_stream(stream));
}

int64_t gq_inv_chol_workspace_size(int64_t n) {
  return n <= 0 ? 256 : gq::inv_chol_scratch_floats(n) * (int64_t)sizeof(float) + 256;
}

int gq_inv_chol(float* a, int64_t n, int64_t lda, void* workspace, int64_t workspace_bytes,
                int* status, void* stream) {
  GQ_REQUIRE(a != nullptr && status != nullptr, "gq_inv_chol: NULL a or status");
  GQ_REQUIRE(n > 0 && lda >= n, "gq_inv_chol: bad shape");
  GQ_REQUIRE(workspace_bytes >= gq_inv_chol_workspace_size(n), "gq_inv_chol: workspace too small");
  GQ_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
             "gq_inv_chol: workspace must be 256-byte aligned");
  GQ_TRY(gq::diag_kernel_setup());
  return gq::inv_chol(a, n, lda, static_cast<float*>(workspace), status, gq::as_stream(stream));
}

int gq_hessian_prepare(const float* h, int64_t d, int64_t ldh, const int32_t* perm,
                       double damp_percent, int attempt, float* b, float* hd_out, float* mean,
                       void* stream) {
  GQ_REQUIRE(h != nullptr && b != nullptr && mean != nullptr, "gq_hessian_prepare: NULL argument");
  GQ_REQUIRE(d > 0 && ldh >= d, "gq_hessian_prepare: bad shape");
  GQ_REQUIRE(damp_percent >= 0.0 && attempt >= 0 && attempt < 5,
             "gq_hessian_prepare: bad damp_percent or attempt");
  GQ_REQUIRE(d * (int64_t)sizeof(float) <= gq::MAX_ROW_BYTES, "gq_hessian_prepare: d = %lld too large",
             (long long)d);
  cudaStream_t st = gq::as_stream(stream);
  GQ_TRY(gq::diag_kernel_setup());
  gq::diag_mean_kernel<<<1, 1024, 0, st>>>(h, d, ldh, mean);
  GQ_TRY(gq::check_launch("diag_mean"));
  const float damp = (float)(std::pow(10.0, attempt) * damp_percent);
  const unsigned rows_grid = (unsigned)std::min<int64_t>(d, 148 * 16);
  const size_t row_bytes = (size_t)d * sizeof(float);
  gq::damp_permute_rows_kernel<true><<<rows_grid, 256, row_bytes, st>>>(h, d, ldh, perm, mean,
                                                                        damp, b);
  GQ_TRY(gq::check_launch("damp_permute"));
  if (hd_out) {
    gq::damp_permute_rows_kernel<false><<<rows_grid, 256, row_bytes, st>>>(h, d, ldh, perm, mean,
                                                                           damp, hd_out);
    GQ_TRY(gq::check_launch("damp_permute"));
  }
  return GQ_OK;
}

int gq_reverse_lower(const float* x, int64_t d, int64_t ldx, float* u, int64_t ldu, void* stream) {
  GQ_REQUIRE(x != nullptr && u != nullptr && d > 0 && ldx >= d && ldu >= d,
             "gq_reverse_lower: bad argument");
  cudaStream_t st = gq::as_stream(stream);
  gq::reverse_copy_kernel<<<(unsigned)std::min<int64_t>(d, 148 * 16), 256, 0, st>>>(x, d, ldx, u,
                                                                                   ldu);
  return gq::check_launch("reverse_copy");
}

int gq_sgemm_tri(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, float alpha,
                 const float* a, int64_t lda, const float* b, int64_t ldb, float beta, float* c,
                 int64_t ldc, int tri, void* stream) {
  GQ_REQUIRE(tri >= 0 && tri <= 4, "gq_sgemm_tri: tri must be 0..4");
  GQ_REQUIRE(M >= 0 && N >= 0 && K >= 0, "gq_sgemm_tri: negative shape");
  return gq::sgemm_tri(trans_a, trans_b, M, N, K, alpha, a, lda, b, ldb, beta, c, ldc, tri,
                       gq::as_stream(stream));
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
  float* ht = ws;                                   // d*d
  float* scratch = ht + gq::hessian_scratch_offset(d);     // inv_chol_scratch_floats(d)
  float* mean = scratch + gq::inv_chol_scratch_floats(d);  // 1 float
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
  GQ_TRY(gq::inv_chol(ht, d, d, scratch, status, st));
  gq::reverse_copy_kernel<<<rows_grid, 256, 0, st>>>(ht, d, d, u, ldu);
  return gq::check_launch("reverse_copy");
}

int64_t gq_factor_from_x_workspace_size(int64_t tokens, int64_t d) {
  return gq::factor_x_gather_offset(d) + tokens * d * 2;
}

int gq_factor_from_x_attempt(const uint16_t* x, int64_t tokens, int64_t d, int64_t ldx,
                             int ordering, double damp_percent, int reserve_sms, float* u,
                             int64_t ldu, int32_t* perm, void* workspace, int64_t workspace_bytes,
                             int* status, void* stats_stream, void* chain_stream) {
  GQ_REQUIRE(x != nullptr && u != nullptr && perm != nullptr && status != nullptr,
             "gq_factor_from_x_attempt: NULL x, u, perm or status");
  GQ_REQUIRE(tokens > 0 && d > 0 && ldx >= d && ldu >= d, "gq_factor_from_x_attempt: bad shape");
  GQ_REQUIRE(d % 8 == 0 && ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
             "gq_factor_from_x_attempt: d and ldx must be multiples of 8 and x 16-byte aligned");
  GQ_REQUIRE(ordering == 0 || ordering == 1, "gq_factor_from_x_attempt: ordering must be 0 or 1");
  GQ_REQUIRE(damp_percent >= 0.0, "gq_factor_from_x_attempt: negative damp_percent");
  GQ_REQUIRE(reserve_sms >= 0, "gq_factor_from_x_attempt: negative reserve_sms");
  GQ_REQUIRE(workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0 &&
                 workspace_bytes >= gq_factor_from_x_workspace_size(tokens, d),
             "gq_factor_from_x_attempt: workspace must be 256-byte aligned and hold %lld bytes",
             (long long)gq_factor_from_x_workspace_size(tokens, d));
  const size_t gather_smem = (size_t)((d * 4 + 15) / 16) * 16 + (size_t)d * 2;
  GQ_REQUIRE(gather_smem <= (size_t)gq::MAX_ROW_BYTES, "gq_factor_from_x_attempt: d = %lld too large",
             (long long)d);
  cudaStream_t ss = gq::as_stream(stats_stream), cs = gq::as_stream(chain_stream);
  float* ws = reinterpret_cast<float*>(workspace);
  float* ht = ws;
  float* scratch = ht + gq::hessian_scratch_offset(d);
  float* mean = scratch + gq::inv_chol_scratch_floats(d);
  uint16_t* xr = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(workspace) +
                                             gq::factor_x_gather_offset(d));
  GQ_TRY(gq::diag_kernel_setup());
  static int gather_attr_device = -1;
  int dev = 0;
  GQ_CHECK_CUDA(cudaGetDevice(&dev));
  if (gather_attr_device != dev) {
    GQ_CHECK_CUDA(cudaFuncSetAttribute(gq::gather_cols_reversed_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       gq::MAX_ROW_BYTES));
    gather_attr_device = dev;
  }
  gq::Forks* forks = nullptr;
  GQ_TRY(gq::forks_for(cs, &forks));
  cudaEvent_t ev_a11 = forks->a11_ready, ev_all = forks->h_ready;
  // statistics stream: diagonal tiles of H in original order -> perm, mean;
  // gathered columns; A11, then A21 and A22 with reserve_sms left to the chain
  GQ_TRY(gq::tc::launch(x, ldx, x, ldx, tokens, d, d, ht, d, 0, 1, ss, 1));
  GQ_TRY(gq::act_order_perm(ht, d, d, ordering, perm, ss));
  gq::diag_mean_kernel<<<1, 1024, 0, ss>>>(ht, d, d, mean);
  GQ_TRY(gq::check_launch("diag_mean"));
  const unsigned rows_grid = (unsigned)std::min<int64_t>(tokens, 148 * 8);
  gq::gather_cols_reversed_kernel<<<rows_grid, 256, gather_smem, ss>>>(x, tokens, d, ldx, perm,
                                                                       xr);
  GQ_TRY(gq::check_launch("gather_cols_reversed"));
  const float damp = (float)damp_percent;
  const int64_t n1 = d > gq::NB ? gq::split_n1(d) : d, n2 = d - n1;
  GQ_TRY(gq::tc::launch(xr, d, xr, d, tokens, n1, n1, ht, d, 0, 1, ss, 0));
  GQ_TRY(gq::lower_damped_from_upper(ht, n1, d, mean, damp, ss));
  if (n2 > 0) GQ_CHECK_CUDA(cudaMemset2DAsync(ht + n1, d * 4, 0, n2 * 4, n1, ss));
  GQ_CHECK_CUDA(cudaMemsetAsync(status, 0, sizeof(int), ss));
  GQ_CHECK_CUDA(cudaEventRecord(ev_a11, ss));
  if (n2 > 0) {
    const int prev = gq::cta_budget();
    const int keep = std::max(1, std::min(prev, gq::sm_count() - reserve_sms));
    gq_set_cta_budget(keep);
    int rc = gq::tc::launch(xr + n1, d, xr, d, tokens, n2, n1, ht + n1 * d, d, 0, 0, ss, 0);
    if (rc == GQ_OK) rc = gq::tc::launch(xr + n1, d, xr + n1, d, tokens, n2, n2, ht + n1 * d + n1,
                                         d, 0, 1, ss, 0);
    gq_set_cta_budget(prev == gq::sm_count() ? 0 : prev);
    GQ_TRY(rc);
    GQ_TRY(gq::lower_damped_from_upper(ht + n1 * d + n1, n2, d, mean, damp, ss));
  }
  GQ_CHECK_CUDA(cudaEventRecord(ev_all, ss));
  // chain stream: rec(A11) as soon as A11 is formed, the rest once H is
  GQ_CHECK_CUDA(cudaStreamWaitEvent(cs, ev_a11, 0));
  GQ_TRY(gq::inv_chol_rec(ht, n1, d, scratch, status, cs, forks, 1));
  GQ_CHECK_CUDA(cudaStreamWaitEvent(cs, ev_all, 0));
  if (n2 > 0) GQ_TRY(gq::inv_chol_after_a11(ht, d, d, scratch, status, cs, forks, 0));
  gq::reverse_copy_kernel<<<(unsigned)std::min<int64_t>(d, 148 * 16), 256, 0, cs>>>(ht, d, d, u,
                                                                                     ldu);
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
  float* mean = ws + gq::hessian_scratch_offset(d) + gq::inv_chol_scratch_floats(d);
  int* status = reinterpret_cast<int*>(mean + 16);           // 1 int
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
