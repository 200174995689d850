// Symmetric eigendecomposition for process_hessian's eigh branch
// (gptq_ref.py:95-99 calls jnp.linalg.eigh): cyclic two-sided Jacobi with
// the parallel round-robin ordering (Brent & Luk, 1985).
//
// With N = n rounded up to even, each sweep has N - 1 rounds; a round pairs
// all N indices into N/2 disjoint pairs (the "circle" schedule: index 0 stays,
// the others rotate by one place per round), so its N/2 plane rotations
// commute and are applied together:
//   1. params_kernel: for every pair (p, q) the symmetric Schur rotation
//      (Golub & Van Loan, Algorithm 8.4.1) that zeroes a_pq, computed in
//      float64 from the round's a_pp, a_qq, a_pq; skipped (identity) when
//      |a_pq| <= tol * sqrt(|a_pp a_qq|);
//   2. rows_kernel: A <- J^T A, one CTA per pair updates rows p and q;
//   3. cols_kernel: A <- A J and V <- V J, one warp per row: the row is staged
//      in shared memory and every element combined with its pair partner.
// A sweep without a single rotation ends the iteration.  The eigenvalues are
// the final diagonal; they are sorted ascending (the order eigh returns, ties
// by index) and V's columns gathered to match.
//
// All kernels are stream-ordered; no kernel waits on another.  The host reads
// one rotation count per sweep (the entry point is blocking).
#include "gq_common.cuh"

#include <cfloat>

namespace gq {
namespace eig {

// Position k (0..N-1) of the circle schedule in round r -> index.
__device__ __forceinline__ int64_t circle_index(int64_t k, int64_t r, int64_t N) {
  return k == 0 ? 0 : ((k - 1 + r) % (N - 1)) + 1;
}
// index -> position in round r.
__device__ __forceinline__ int64_t circle_pos(int64_t idx, int64_t r, int64_t N) {
  return idx == 0 ? 0 : (((idx - 1 - r) % (N - 1)) + (N - 1)) % (N - 1) + 1;
}

__global__ void params_kernel(const float* __restrict__ a, int64_t n, int64_t lda, int64_t N,
                              int64_t r, float tol, float2* __restrict__ cs,
                              int* __restrict__ rotations) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= N / 2) return;
  int64_t p = circle_index(i, r, N), q = circle_index(N - 1 - i, r, N);
  if (p > q) {
    const int64_t t = p;
    p = q;
    q = t;
  }
  float2 out = make_float2(1.f, 0.f);
  if (q < n) {
    const double app = a[p * lda + p], aqq = a[q * lda + q], apq = a[p * lda + q];
    if (apq != 0.0 && fabs(apq) > (double)tol * sqrt(fabs(app * aqq))) {
      const double tau = (aqq - app) / (2.0 * apq);
      const double t = (tau >= 0.0 ? 1.0 : -1.0) / (fabs(tau) + sqrt(1.0 + tau * tau));
      const double c = 1.0 / sqrt(1.0 + t * t);
      out = make_float2((float)c, (float)(t * c));
      atomicAdd(rotations, 1);
    }
  }
  cs[i] = out;
}

// A <- J^T A: rows p, q of the pair handled by this CTA.
__global__ void rows_kernel(float* __restrict__ a, int64_t n, int64_t lda, int64_t N, int64_t r,
                            const float2* __restrict__ cs) {
  const int64_t i = blockIdx.x;
  const float2 g = cs[i];
  if (g.x == 1.f && g.y == 0.f) return;
  int64_t p = circle_index(i, r, N), q = circle_index(N - 1 - i, r, N);
  if (p > q) {
    const int64_t t = p;
    p = q;
    q = t;
  }
  float* rp = a + p * lda;
  float* rq = a + q * lda;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
    const float x = rp[j], y = rq[j];
    rp[j] = g.x * x - g.y * y;
    rq[j] = g.y * x + g.x * y;
  }
}

// M <- M J for the rows of A (rows 0..n-1) and of V (rows n..2n-1), one warp
// per row, the row staged in shared memory (rows_per_cta x n floats).
__global__ void cols_kernel(float* __restrict__ a, int64_t lda, float* __restrict__ v, int64_t ldv,
                            int64_t n, int64_t N, int64_t r, const float2* __restrict__ cs) {
  extern __shared__ float srow[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + warp;
  if (row >= 2 * n) return;
  float* m = row < n ? a + row * lda : v + (row - n) * ldv;
  float* s = srow + (int64_t)warp * n;
  for (int64_t j = lane; j < n; j += 32) s[j] = m[j];
  __syncwarp();
  for (int64_t j = lane; j < n; j += 32) {
    const int64_t k = circle_pos(j, r, N);
    const int64_t pair = k < N / 2 ? k : N - 1 - k;
    const int64_t partner = circle_index(N - 1 - k, r, N);
    if (partner >= n) continue;  // paired with the padding index: untouched
    const float2 g = cs[pair];
    if (g.x == 1.f && g.y == 0.f) continue;
    if (row == partner) {  // the entry (p, q) the rotation annihilates
      m[j] = 0.f;
      continue;
    }
    // within the pair the smaller index plays p, the larger q
    if (j < partner) m[j] = g.x * s[j] - g.y * s[partner];
    else m[j] = g.y * s[partner] + g.x * s[j];
  }
}

__global__ void init_v_kernel(float* __restrict__ v, int64_t n, int64_t ldv) {
  const int64_t i = blockIdx.y;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x)
    v[i * ldv + j] = (i == j) ? 1.f : 0.f;
}

__global__ void copy_rows_kernel(const float* __restrict__ src, int64_t lds, float* __restrict__ dst,
                                 int64_t ldd, int64_t n) {
  const int64_t i = blockIdx.y;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x)
    dst[i * ldd + j] = src[i * lds + j];
}

// Ascending order of the diagonal: rank_i = #{d_j < d_i} + #{d_j == d_i, j < i}.
__global__ void sort_rank_kernel(const float* __restrict__ a, int64_t n, int64_t lda,
                                 float* __restrict__ w, int32_t* __restrict__ order) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float di = a[i * lda + i];
  int64_t rank = 0;
  for (int64_t j = 0; j < n; ++j) {
    const float dj = a[j * lda + j];
    rank += (dj < di) || (dj == di && j < i);
  }
  w[rank] = di;
  order[rank] = (int32_t)i;
}

// vout[:, k] = v[:, order[k]], one CTA per row of V.
__global__ void gather_cols_kernel(const float* __restrict__ v, int64_t ldv,
                                   const int32_t* __restrict__ order, int64_t n,
                                   float* __restrict__ vout, int64_t ldo) {
  const int64_t i = blockIdx.x;
  for (int64_t k = threadIdx.x; k < n; k += blockDim.x) vout[i * ldo + k] = v[i * ldv + order[k]];
}

inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

}  // namespace eig
}  // namespace gq

extern "C" {

int64_t gq_syevj_workspace_size(int64_t n) {
  using gq::eig::align256;
  if (n <= 0) return 256;
  const int64_t N = n + (n & 1);
  return align256(n * n * 4) * 2 + align256(N / 2 * 8) + align256(n * 4) + 256;
}

int gq_syevj(const float* a, int64_t n, int64_t lda, float* w, float* v, int64_t ldv,
             int max_sweeps, int* sweeps_done, void* workspace, int64_t workspace_bytes,
             void* stream) {
  using namespace gq;
  using namespace gq::eig;
  GQ_REQUIRE(n >= 0 && lda >= n && ldv >= n, "gq_syevj: bad shape");
  GQ_REQUIRE(n == 0 || (a != nullptr && w != nullptr && v != nullptr), "gq_syevj: NULL argument");
  GQ_REQUIRE(max_sweeps >= 1 && max_sweeps <= 100, "gq_syevj: max_sweeps must be in [1, 100]");
  GQ_REQUIRE(n <= (200 * 1024) / 4, "gq_syevj: n=%lld exceeds the staged row (at most 51200)",
             (long long)n);
  GQ_REQUIRE(workspace_bytes >= gq_syevj_workspace_size(n), "gq_syevj: workspace too small");
  GQ_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
             "gq_syevj: workspace must be 256-byte aligned");
  if (sweeps_done) *sweeps_done = 0;
  if (n == 0) return GQ_OK;
  cudaStream_t st = as_stream(stream);
  char* ws = static_cast<char*>(workspace);
  float* aw = reinterpret_cast<float*>(ws);                       // working copy of A [n, n]
  float* vw = reinterpret_cast<float*>(ws + align256(n * n * 4));  // V before sorting [n, n]
  float2* cs = reinterpret_cast<float2*>(ws + 2 * align256(n * n * 4));
  int32_t* order = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(cs) +
                                              align256(((n + (n & 1)) / 2) * 8));
  int* rot = reinterpret_cast<int*>(reinterpret_cast<char*>(order) + align256(n * 4));
  const int64_t N = n + (n & 1);
  const dim3 rowsgrid((unsigned)std::min<int64_t>(ceil_div(n, 256), 64), (unsigned)n);
  copy_rows_kernel<<<rowsgrid, 256, 0, st>>>(a, lda, aw, n, n);
  GQ_TRY(check_launch("syevj copy"));
  init_v_kernel<<<rowsgrid, 256, 0, st>>>(vw, n, n);
  GQ_TRY(check_launch("syevj init"));
  // rows staged per CTA in cols_kernel
  const int rows_per_cta = (int)std::max<int64_t>(1, std::min<int64_t>(8, (200 * 1024) / (4 * n)));
  const size_t smem = (size_t)rows_per_cta * n * 4;
  GQ_CHECK_CUDA(cudaFuncSetAttribute(cols_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)std::max<size_t>(smem, 48 * 1024)));
  const float tol = 4.f * FLT_EPSILON;
  int sweep = 0;
  if (n > 1) {
    for (sweep = 0; sweep < max_sweeps; ++sweep) {
      GQ_CHECK_CUDA(cudaMemsetAsync(rot, 0, sizeof(int), st));
      for (int64_t r = 0; r < N - 1; ++r) {
        params_kernel<<<(unsigned)ceil_div(N / 2, 128), 128, 0, st>>>(aw, n, n, N, r, tol, cs, rot);
        GQ_TRY(check_launch("syevj params"));
        rows_kernel<<<(unsigned)(N / 2), 256, 0, st>>>(aw, n, n, N, r, cs);
        GQ_TRY(check_launch("syevj rows"));
        cols_kernel<<<(unsigned)ceil_div(2 * n, rows_per_cta), 32 * rows_per_cta, smem, st>>>(
            aw, n, vw, n, n, N, r, cs);
        GQ_TRY(check_launch("syevj cols"));
      }
      int host_rot = 0;
      GQ_CHECK_CUDA(cudaMemcpyAsync(&host_rot, rot, sizeof(int), cudaMemcpyDeviceToHost, st));
      GQ_CHECK_CUDA(cudaStreamSynchronize(st));
      if (host_rot == 0) {
        ++sweep;
        break;
      }
    }
  }
  if (sweeps_done) *sweeps_done = sweep;
  sort_rank_kernel<<<(unsigned)ceil_div(n, 128), 128, 0, st>>>(aw, n, n, w, order);
  GQ_TRY(check_launch("syevj sort"));
  gather_cols_kernel<<<(unsigned)n, 256, 0, st>>>(vw, n, order, n, v, ldv);
  return check_launch("syevj gather");
}

}  // extern "C"
