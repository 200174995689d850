// Blocked column-pivoted Householder QR (pallas/blocked_pivoted_qr.py).
//
// Working copy: the matrix transposed into column-major order, at[c][r]
// (ld = m), so pivot columns, swaps, Householder vectors and column norms are
// contiguous.  Per panel of P columns starting at k:
//   * one "step" kernel per pivot, on a cluster of eight CTAs that split the
//     column's rows: choose the pivot from the norm metadata, swap whole
//     columns, form the reflector, append it to the compact WY pair
//     (yt = Y^T, P x (m-k); T, P x P) and produce the vector
//     left = (y_r T^T) Y^T that exposes row r of the transformed trailing
//     block;
//   * one all-SM "exposed row" kernel: e_c = B[r][c] - left . B[:, c] for the
//     deferred (stale) trailing columns, and the norm downdate
//     norms_c = max(norms_c - e_c^2, 0) -- the BLAS-2 pass that reads the
//     whole trailing block every step;
//   * at the panel end the compact-WY update B <- B - Y (T^T (Y^T B)) (two
//     tensor-core fp32 GEMMs around a small T application) and an exact norm
//     refresh from rows >= panel end.
//
// semantics = 0 ("reference") reproduces _factor_panel_compiled
// (:1479-1589) and the driver (:1627-1722) exactly, including:
//   * pivots chosen among all columns >= j, deferred trailing ones too;
//   * panel columns updated eagerly, their norms downdated by the new row and
//     recomputed exactly every 8 steps (:1014-1104);
//   * the reflector built from column j - k of a[k:, :] (the panel-local
//     index reused as a column index, :359-366);
//   * the exposed row taken at panel-local row j (the global index reused,
//     :1106-1112), clamped like dynamic_index_in_dim;
//   * panels starting every P columns even after a "smallest" early stop.
// semantics = 1 ("intended") is a correct blocked QRCP (the BLAS-3 scheme of
// Quintana-Orti, Sun & Bischof, 1998): every column >= j is deferred, the
// chosen pivot column is brought up to date with the panel's reflectors
// before its Householder vector is formed, the true exposed row j downdates
// all remaining norms, and a panel ends early when a downdated norm has lost
// too much of its reference value to be trusted (the LAPACK xLAQPS rule),
// after which the next panel starts from exact norms.  Its pivots and R equal
// unblocked Householder QRCP in exact arithmetic.
#include "gq_common.cuh"

#include <algorithm>
#include <vector>

namespace gq {

int sgemm(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
          const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int uplo, cudaStream_t st);

namespace qr {

constexpr float ZERO_TOL_SQ = 1e-24f;  // ZERO_TOL ** 2 (:52-53)
constexpr int MAX_P = 256;             // widest panel (reference semantics honour panel_size)
constexpr int INTENDED_P = 64;         // panel width used by the intended (exact) factorization

// Device control block, one per factorization.
struct Ctrl {
  int active;     // accepted reflectors in the current panel
  int done;       // panel stopped ("smallest" with no mass left, or early end)
  int early_end;  // intended: a norm downdate lost precision -> end after this step
  int row_sel;    // panel-local row exposed by the current step
};

__global__ void transpose_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                                 int64_t lds, float* __restrict__ dst, int64_t ldd) {
  __shared__ float tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * lds + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) dst[c * ldd + r] = tile[threadIdx.x][i];
  }
}

// norms[c] = sum_{r >= r0} at[c][r]^2 (warp per column); r0 >= m gives zeros.
__global__ void col_sqnorms_kernel(const float* __restrict__ at, int64_t m, int64_t n, int64_t r0,
                                   float* __restrict__ norms, float* __restrict__ copy) {
  const int lane = threadIdx.x & 31;
  const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (c >= n) return;
  float s = 0.f;
  for (int64_t r = r0 + lane; r < m; r += 32) {
    float v = at[c * m + r];
    s = fmaf(v, v, s);
  }
  s = warp_sum(s);
  if (lane == 0) {
    norms[c] = s;
    if (copy) copy[c] = s;
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (lane < (int)(blockDim.x >> 5)) ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;  // valid in every thread
}

// (value, index) best with the first-index tie rule; larger = true -> argmax.
__device__ __forceinline__ void better(float& bv, int& bi, float v, int i, bool larger) {
  bool take = larger ? (v > bv || (v == bv && i < bi)) : (v < bv || (v == bv && i < bi));
  if (take) {
    bv = v;
    bi = i;
  }
}

__device__ int block_arg(float v, int i, bool larger, float* redv, int* redi) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, i, o);
    better(v, i, ov, oi, larger);
  }
  __syncthreads();
  if (lane == 0) {
    redv[warp] = v;
    redi[warp] = i;
  }
  __syncthreads();
  if (warp == 0) {
    float w = (lane < (int)(blockDim.x >> 5)) ? redv[lane] : (larger ? -INFINITY : INFINITY);
    int wi = (lane < (int)(blockDim.x >> 5)) ? redi[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, w, o);
      int oi = __shfl_xor_sync(0xffffffffu, wi, o);
      better(w, wi, ov, oi, larger);
    }
    if (lane == 0) redi[0] = wi;
  }
  __syncthreads();
  return redi[0];
}

struct StepArgs {
  float* at;       // n x m column-major working copy
  int64_t m, n;
  int64_t k;       // panel start
  int64_t pe;      // nominal panel end
  int64_t j;       // global step index
  int P;           // panel width (yt rows / T size)
  float* yt;       // P x (m - k): reflector i in row i (panel-local rows)
  float* t;        // P x P
  float* tau;      // P
  float* norms;    // n
  float* normref;  // n: exact norms at the panel start (intended semantics)
  int32_t* perm;   // n
  float* left;     // m - k
  Ctrl* ctrl;
  int smallest;
  int nopivot;     // unpivoted Householder QR: the pivot of step j is column j
  int semantics;   // 0 reference, 1 intended
};

// ---------------------------------------------------------------------------
// The pivot step on a cluster of CL CTAs.  The step's L-long vectors (the
// pivot column, the reflector v, the rows of Y^T) are split into CL row
// slices, one per CTA, so the four passes over Y^T a step makes (Y^T col,
// Y z, Y^T v, left = s Y^T) read L2 through CL SMs instead of one.  Dot
// products are formed per slice and summed across the cluster through
// distributed shared memory in rank order, so every CTA holds the same sums;
// the small P-sized work (pivot choice, T, the exposed-row weights) is done
// redundantly in every CTA and written once.  Compared with doing the step
// in one CTA, only the grouping of the L-long sums differs.
constexpr int CL = 8;            // CTAs per cluster (portable size)
constexpr int CT = 512;          // threads per CTA
constexpr int CTW = CT / 32;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ float ld_cluster(const float* local, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_addr(local)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ int64_t i64min(int64_t x, int64_t y) { return x < y ? x : y; }
__device__ __forceinline__ int64_t i64max(int64_t x, int64_t y) { return x > y ? x : y; }
__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Double-buffered partial vectors: each CTA writes its partials into
// part[buf], the cluster synchronizes, and every CTA sums the CL partial
// vectors in rank order into out.  A buffer is written again only two
// reductions later, after every CTA has passed the barrier that follows its
// reads.  buf is a per-thread copy, flipped in step by every thread.
__device__ void cluster_sum(float (*part)[MAX_P + 8], int& buf, int count, float* out) {
  cluster_barrier();
  const float* src = part[buf];
  for (int t = threadIdx.x; t < count; t += blockDim.x) {
    float s = ld_cluster(src + t, 0);
    for (uint32_t q = 1; q < CL; ++q) s = __fadd_rn(s, ld_cluster(src + t, q));
    out[t] = s;
  }
  __syncthreads();
  buf ^= 1;
}

__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(CT)
qr_step_cluster_kernel(StepArgs a) {
  // launched as a programmatic dependent of the previous kernel: wait for it
  // to complete, then let the next kernel be scheduled behind this one
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ __align__(16) float sm[];
  __shared__ float redv[CTW];
  __shared__ int redi[CTW];
  __shared__ float sw[MAX_P + 1];
  __shared__ float sw2[MAX_P + 1];
  __shared__ float sums[MAX_P + 8];
  __shared__ float part[2][MAX_P + 8];
  __shared__ int s_flag;

  Ctrl* ctrl = a.ctrl;
  if (ctrl->done) return;
  if (a.semantics == 1 && ctrl->early_end) {
    if (cta_rank() == 0 && threadIdx.x == 0) ctrl->done = 1;
    return;
  }
  const int64_t m = a.m, n = a.n, k = a.k, j = a.j, pe = a.pe;
  const int64_t L = m - k;
  const int lj = (int)(j - k);
  const int P = a.P;
  const uint32_t rank = cta_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // this CTA's rows [r0, r1) of the panel-local range [0, L)
  const int64_t Ls = (L + CL - 1) / CL;
  const int64_t r0 = i64min(L, (int64_t)rank * Ls), r1 = i64min(L, r0 + Ls);
  float* v = sm;        // v[r - r0]
  float* col = sm + Ls;  // col[r - r0]
  int buf = 0;

  // 1. "smallest": stop when no remaining norm exceeds ZERO_TOL^2 (every CTA alike)
  if (a.smallest) {
    int any = 0;
    for (int64_t c = j + tid; c < n; c += blockDim.x) any |= (a.norms[c] > ZERO_TOL_SQ);
    if (tid == 0) s_flag = 0;
    __syncthreads();
    if (any) atomicOr(&s_flag, 1);
    __syncthreads();
    if (!s_flag) {
      if (rank == 0 && tid == 0) ctrl->done = 1;
      return;
    }
  }
  // 2. pivot: first argmax / argmin over columns >= j (every CTA alike)
  int p = (int)j;
  if (!a.nopivot) {
    const bool larger = !a.smallest;
    float bv = larger ? -INFINITY : INFINITY;
    int bi = 0x7fffffff;
    for (int64_t c = j + tid; c < n; c += blockDim.x) {
      float x = a.norms[c];
      if (a.smallest && !(x > ZERO_TOL_SQ)) x = INFINITY;
      better(bv, bi, x, (int)c, larger);
    }
    p = block_arg(bv, bi, larger, redv, redi);
    if (p == 0x7fffffff) p = (int)j;
  }
  // every CTA has read the norms before CTA 0 swaps two of them (the
  // intended factorization reads no norm later in the step, so there the
  // scalar swap waits until the end and needs no barrier here)
  if (a.semantics == 0) cluster_barrier();
  // 3. swap whole columns j and p: this CTA's slice of rows [k, m) and a share of [0, k)
  if (p != j) {
    float* cj = a.at + j * m;
    float* cp = a.at + (int64_t)p * m;
    for (int64_t r = k + r0 + tid; r < k + r1; r += blockDim.x) {
      float x = cj[r];
      cj[r] = cp[r];
      cp[r] = x;
    }
    const int64_t ks = (k + CL - 1) / CL;
    for (int64_t r = i64min(k, rank * ks) + tid; r < i64min(k, (rank + 1) * ks);
         r += blockDim.x) {
      float x = cj[r];
      cj[r] = cp[r];
      cp[r] = x;
    }
  }
  auto swap_scalars = [&]() {
    if (p != j && rank == 0 && tid == 0) {
      int32_t tp = a.perm[j];
      a.perm[j] = a.perm[p];
      a.perm[p] = tp;
      float tn = a.norms[j];
      a.norms[j] = a.norms[p];
      a.norms[p] = tn;
      if (a.normref) {
        float tr = a.normref[j];
        a.normref[j] = a.normref[p];
        a.normref[p] = tr;
      }
    }
  };
  if (a.semantics == 0) swap_scalars();
  __syncthreads();

  // 4. the column the reflector is built from (this CTA's rows)
  const int64_t src = (a.semantics == 0) ? (j - k) : j;
  for (int64_t r = r0 + tid; r < r1; r += blockDim.x) col[r - r0] = a.at[src * m + k + r];
  __syncthreads();
  if (a.semantics == 1 && lj > 0) {
    // bring the deferred pivot column up to date: col -= Y (T^T (Y^T col))
    for (int i = warp; i < lj; i += CTW) {
      const float* yi = a.yt + (int64_t)i * L;
      float s = 0.f;
      for (int64_t r = r0 + lane; r < r1; r += 32) s = fmaf(yi[r], col[r - r0], s);
      s = warp_sum(s);
      if (lane == 0) part[buf][i] = s;
    }
    cluster_sum(part, buf, lj, sums);
    if (tid < lj) {
      float z = 0.f;
      for (int l = 0; l <= tid; ++l) z = fmaf(a.t[l * P + tid], sums[l], z);
      sw2[tid] = z;
    }
    __syncthreads();
    for (int64_t r = r0 + tid; r < r1; r += blockDim.x) {
      float s = 0.f;
      for (int i = 0; i < lj; ++i) s = fmaf(a.yt[(int64_t)i * L + r], sw2[i], s);
      col[r - r0] = col[r - r0] - s;
    }
    __syncthreads();
  }
  // Householder vector: sigma over rows below lj; x0 = col[lj] from its owner
  {
    float mine = 0.f;
    for (int64_t r = i64max(r0, lj + 1) + tid; r < r1; r += blockDim.x)
      mine = fmaf(col[r - r0], col[r - r0], mine);
    const float blk = block_sum(mine, redv);
    if (tid == 0) {
      part[buf][0] = blk;
      part[buf][1] = (lj >= r0 && lj < r1) ? col[lj - r0] : 0.f;
    }
  }
  cluster_barrier();
  float sigma, x0;
  {
    const float* src_part = part[buf];
    sigma = ld_cluster(src_part, 0);
    for (uint32_t q = 1; q < CL; ++q) sigma = __fadd_rn(sigma, ld_cluster(src_part, q));
    x0 = ld_cluster(src_part + 1, (uint32_t)(lj / Ls));
  }
  __syncthreads();
  buf ^= 1;
  float tau_j, alpha, beta = 1.f;
  if (sigma == 0.f) {
    tau_j = 0.f;
    alpha = x0;
  } else {
    float nx = sqrtf(__fadd_rn(__fmul_rn(x0, x0), sigma));
    alpha = (x0 <= 0.f) ? nx : -nx;
    beta = __fsub_rn(x0, alpha);
    tau_j = __fdiv_rn(-beta, alpha);
  }
  for (int64_t r = r0 + tid; r < r1; r += blockDim.x) {
    float vr;
    if (r == lj) vr = 1.f;
    else if (r < lj || sigma == 0.f) vr = 0.f;
    else vr = __fdiv_rn(col[r - r0], beta);
    v[r - r0] = vr;
    a.yt[(int64_t)lj * L + r] = vr;
  }
  __syncthreads();
  // 5. append to T: T[:lj, lj] = T_prev (-tau Y_prev^T v); T[lj, lj] = tau
  if (lj > 0) {
    for (int i = warp; i < lj; i += CTW) {
      const float* yi = a.yt + (int64_t)i * L;
      float s = 0.f;
      for (int64_t r = r0 + lane; r < r1; r += 32) s = fmaf(yi[r], v[r - r0], s);
      s = warp_sum(s);
      if (lane == 0) part[buf][i] = s;
    }
    cluster_sum(part, buf, lj, sums);
    if (tid < lj) sw[tid] = -tau_j * sums[tid];
    __syncthreads();
    if (tid < lj) {
      float s = 0.f;
      for (int l = tid; l < lj; ++l) s = fmaf(a.t[tid * P + l], sw[l], s);
      sw2[tid] = s;
    }
    __syncthreads();
  }
  if (rank == 0) {
    if (tid < lj) a.t[tid * P + lj] = sw2[tid];
    if (tid == 0) {
      a.t[lj * P + lj] = tau_j;
      a.tau[lj] = tau_j;
    }
  }
  __syncthreads();

  if (a.semantics == 0) {
    // 6. eager reflector on panel columns j..pe-1
    const int nc = (int)(pe - j);
    for (int ci = warp; ci < nc; ci += CTW) {
      const float* cc = a.at + (j + ci) * m + k;
      float s = 0.f;
      for (int64_t r = r0 + lane; r < r1; r += 32) s = fmaf(v[r - r0], cc[r], s);
      s = warp_sum(s);
      if (lane == 0) part[buf][ci] = s;
    }
    cluster_sum(part, buf, nc, sums);
    for (int ci = warp; ci < nc; ci += CTW) {
      float* cc = a.at + (j + ci) * m + k;
      const float wc = tau_j * sums[ci];
      for (int64_t r = r0 + lane; r < r1; r += 32)
        cc[r] = __fsub_rn(cc[r], __fmul_rn(v[r - r0], wc));
    }
    __syncthreads();
  }
  // pivot column: alpha on the diagonal, zeros below; in the intended
  // factorization rows k..j-1 take the brought-up-to-date values
  for (int64_t r = r0 + tid; r < r1; r += blockDim.x) {
    if (r >= lj) a.at[j * m + k + r] = (r == lj) ? alpha : 0.f;
    else if (a.semantics == 1) a.at[j * m + k + r] = col[r - r0];
  }
  // reference semantics read other CTAs' rows of the updated panel columns
  // (norm metadata) and an arbitrary row of Y: make them visible; the
  // intended exposed row is row lj, whose Y entries this step are v[lj] = 1
  // and whose new T column every CTA holds in sw2
  if (a.semantics == 0) cluster_barrier();

  const int64_t nxt = j + 1;
  if (a.semantics == 0 && nxt < n && nxt < pe) {
    // 7a. panel-column norm metadata: exact every 8 steps, else downdated
    const bool refresh = ((nxt - k) % 8) == 0;
    const int nc = (int)(pe - nxt);
    if (refresh) {
      for (int ci = warp; ci < nc; ci += CTW) {
        const float* cc = a.at + (nxt + ci) * m + k;
        float s = 0.f;
        for (int64_t r = i64max(r0, nxt - k) + lane; r < r1; r += 32)
          s = fmaf(cc[r], cc[r], s);
        s = warp_sum(s);
        if (lane == 0) part[buf][ci] = s;
      }
      cluster_sum(part, buf, nc, sums);
      if (rank == 0)
        for (int ci = tid; ci < nc; ci += blockDim.x) a.norms[nxt + ci] = sums[ci];
    } else if (rank == 0) {
      for (int ci = tid; ci < nc; ci += blockDim.x) {
        const float row = a.at[(nxt + ci) * m + j];
        a.norms[nxt + ci] = fmaxf(__fsub_rn(a.norms[nxt + ci], __fmul_rn(row, row)), 0.f);
      }
    }
  }
  // 7b. the vector exposing one row of the transformed deferred block
  const bool exposes = (a.semantics == 0) ? (nxt < n && pe < n) : (nxt < n);
  if (exposes) {
    int64_t rs = lj;
    if (a.semantics == 0) rs = (j < 0) ? 0 : ((j > L - 1) ? L - 1 : j);
    if (tid < P) {
      float s = 0.f;
      if (a.semantics == 0) {
        for (int l = 0; l < P; ++l) s = fmaf(a.yt[(int64_t)l * L + rs], a.t[tid * P + l], s);
      } else {
        // rows of Y beyond lj are zero; Y[lj][lj] = 1 and T[:, lj] is sw2 / tau here
        for (int l = 0; l <= lj; ++l) {
          const float y = (l == lj) ? 1.f : a.yt[(int64_t)l * L + rs];
          const float tv = (l < lj) ? a.t[tid * P + l]
                                    : ((tid < lj) ? sw2[tid] : ((tid == lj) ? tau_j : 0.f));
          s = fmaf(y, tv, s);
        }
        for (int l = lj + 1; l < P; ++l) s = fmaf(0.f, 0.f, s);
      }
      sw[tid] = s;  // row_weights = y_r T^T
    }
    __syncthreads();
    for (int64_t r = r0 + tid; r < r1; r += blockDim.x) {
      float s = 0.f;
      for (int i = 0; i < P; ++i) s = fmaf(sw[i], a.yt[(int64_t)i * L + r], s);
      a.left[r] = s;
    }
    if (rank == 0 && tid == 0) ctrl->row_sel = (int)rs;
  }
  if (rank == 0 && tid == 0) ctrl->active = ctrl->active + 1;
  // no CTA leaves while another may still read its shared memory
  cluster_barrier();
  if (a.semantics == 1) swap_scalars();
}

// Exposed-row downdate over deferred columns [c0, n): warp per column.
__global__ void exposed_row_kernel(const float* __restrict__ at, int64_t m, int64_t n, int64_t k,
                                   int64_t c0, const float* __restrict__ left,
                                   float* __restrict__ norms, const float* __restrict__ normref,
                                   Ctrl* ctrl, float tol) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  if (ctrl->done) return;
  const int lane = threadIdx.x & 31;
  const int64_t L = m - k;
  const int rs = ctrl->row_sel;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t c = c0 + (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); c < n;
       c += nw) {
    const float* b = at + c * m + k;
    float s = 0.f;
    int64_t r = lane * 4;
    if ((m & 3) == 0 && (k & 3) == 0) {
      for (; r + 3 < L; r += 128) {
        float4 bv = *reinterpret_cast<const float4*>(b + r);
        float4 lv = *reinterpret_cast<const float4*>(left + r);
        s = fmaf(lv.x, bv.x, s);
        s = fmaf(lv.y, bv.y, s);
        s = fmaf(lv.z, bv.z, s);
        s = fmaf(lv.w, bv.w, s);
      }
    } else {
      for (int64_t q = lane; q < L; q += 32) s = fmaf(left[q], b[q], s);
    }
    s = warp_sum(s);
    if (lane == 0) {
      float e = __fsub_rn(b[rs], s);
      float nv = fmaxf(__fsub_rn(norms[c], __fmul_rn(e, e)), 0.f);
      norms[c] = nv;
      if (normref && nv <= tol * normref[c] && normref[c] > 0.f) atomicExch(&ctrl->early_end, 1);
    }
  }
}

__global__ void reset_ctrl_kernel(Ctrl* ctrl) {
  ctrl->active = 0;
  ctrl->done = 0;
  ctrl->early_end = 0;
  ctrl->row_sel = 0;
}

// V[k + r][k + i] = yt[i][r] for i < w (reflectors in global rows); columns are strided.
__global__ void store_reflectors_kernel(const float* __restrict__ yt, int64_t m, int64_t k, int w,
                                        float* __restrict__ V, int64_t ldv, const float* __restrict__ tau,
                                        float* __restrict__ tau_out) {
  const int64_t L = m - k;
  const int i = blockIdx.y;
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < m; r += (int64_t)gridDim.x * blockDim.x) {
    float x = (r >= k) ? yt[(int64_t)i * L + (r - k)] : 0.f;
    V[r * ldv + k + i] = x;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && tau_out) tau_out[k + i] = tau[i];
}

struct Work {
  float* at;
  float* yt;
  float* t;
  float* tau;
  float* norms;
  float* normref;
  float* left;
  float* z;
  float* z2;
  float* y;
  Ctrl* ctrl;
};

inline int64_t align256(int64_t b) { return (b + 255) & ~int64_t(255); }

int64_t ws_bytes(int64_t m, int64_t n, int P) {
  int64_t b = 0;
  b += align256(n * m * 4);          // at
  b += align256((int64_t)P * m * 4);  // yt
  b += align256((int64_t)P * P * 4);  // t
  b += align256((int64_t)P * 4);      // tau
  b += align256(n * 4) * 2;          // norms, normref
  b += align256(m * 4);              // left
  b += align256(n * (int64_t)P * 4) * 2;  // z, z2
  b += align256(m * (int64_t)P * 4);      // y
  b += align256(sizeof(Ctrl));
  return b;
}

Work carve(void* ws, int64_t m, int64_t n, int P) {
  char* p = reinterpret_cast<char*>(ws);
  Work w;
  w.at = reinterpret_cast<float*>(p); p += align256(n * m * 4);
  w.yt = reinterpret_cast<float*>(p); p += align256((int64_t)P * m * 4);
  w.t = reinterpret_cast<float*>(p); p += align256((int64_t)P * P * 4);
  w.tau = reinterpret_cast<float*>(p); p += align256((int64_t)P * 4);
  w.norms = reinterpret_cast<float*>(p); p += align256(n * 4);
  w.normref = reinterpret_cast<float*>(p); p += align256(n * 4);
  w.left = reinterpret_cast<float*>(p); p += align256(m * 4);
  w.z = reinterpret_cast<float*>(p); p += align256(n * (int64_t)P * 4);
  w.z2 = reinterpret_cast<float*>(p); p += align256(n * (int64_t)P * 4);
  w.y = reinterpret_cast<float*>(p); p += align256(m * (int64_t)P * 4);
  w.ctrl = reinterpret_cast<Ctrl*>(p);
  return w;
}

// B <- B - Y (T^T (Y^T B)) for deferred columns [c0, n), rows k..m-1 (width w).
// zt2[c][i] = sum_{l <= i} T[l][i] z[l][c]   (z: w x nc, ld nc; zt2: nc x w, ld P);
// one thread per (c, i), i = blockIdx.y
__global__ void apply_t_kernel(const float* __restrict__ z, int64_t nc, int w,
                               const float* __restrict__ t, int P, float* __restrict__ zt2) {
  const int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int i = blockIdx.y;
  if (c >= nc) return;
  float s = 0.f;
  for (int l = 0; l <= i; ++l) s = fmaf(z[(int64_t)l * nc + c], t[l * P + i], s);
  zt2[c * P + i] = s;
}

// B <- B - Y (T^T (Y^T B)) on the deferred columns, as two K-major products
// (tensor cores where the shapes allow) around a small T application:
//   Z = Y^T B (w x nc), Zt2 = (T^T Z)^T (nc x w), Bt -= Zt2 Y^T with Y = yt^T.
int apply_panel(Work& W, int64_t m, int64_t n, int64_t k, int w, int P, int64_t c0,
                cudaStream_t st) {
  if (c0 >= n || w <= 0) return GQ_OK;
  const int64_t L = m - k, nc = n - c0;
  float* bt = W.at + c0 * m + k;  // nc x L, ld m
  GQ_TRY(sgemm(0, 1, w, nc, L, 1.f, W.yt, L, bt, m, 0.f, W.z, nc, 0, st));
  apply_t_kernel<<<dim3((unsigned)ceil_div(nc, 128), (unsigned)w), 128, 0, st>>>(W.z, nc, w, W.t,
                                                                                P, W.z2);
  GQ_TRY(check_launch("apply_t"));
  // y = yt^T: L x w, ld P
  transpose_kernel<<<dim3((unsigned)ceil_div(L, 32), (unsigned)ceil_div(w, 32)), dim3(32, 8), 0,
                     st>>>(W.yt, w, L, L, W.y, P);
  GQ_TRY(check_launch("transpose_y"));
  return sgemm(0, 1, nc, L, w, -1.f, W.z2, P, W.y, P, 1.f, bt, m, 0, st);
}

int norms_from(Work& W, int64_t m, int64_t n, int64_t r0, bool keep_ref, cudaStream_t st) {
  col_sqnorms_kernel<<<(unsigned)ceil_div(n, 8), 256, 0, st>>>(W.at, m, n, r0, W.norms,
                                                               keep_ref ? W.normref : nullptr);
  return check_launch("col_sqnorms");
}

// One panel from k; returns the realized width through *width (host-synced).
int factor_panel(Work& W, int64_t m, int64_t n, int64_t k, int P, int smallest, int semantics,
                 int32_t* perm, cudaStream_t st, int* width) {
  const int64_t limit = std::min(m, n);
  const int64_t pe = std::min(k + (int64_t)P, limit);
  const int64_t L = m - k;
  GQ_CHECK_CUDA(cudaMemsetAsync(W.yt, 0, (size_t)P * L * 4, st));
  GQ_CHECK_CUDA(cudaMemsetAsync(W.t, 0, (size_t)P * P * 4, st));
  GQ_CHECK_CUDA(cudaMemsetAsync(W.tau, 0, (size_t)P * 4, st));
  reset_ctrl_kernel<<<1, 1, 0, st>>>(W.ctrl);
  GQ_TRY(check_launch("reset_ctrl"));
  const int gemv_blocks = std::max(1, sm_count() * 4);
  const float tol3z = 0.000244140625f;  // sqrt(2^-24): LAPACK's xLAQPS recompute threshold
  for (int64_t j = k; j < pe; ++j) {
    StepArgs a;
    a.at = W.at; a.m = m; a.n = n; a.k = k; a.pe = pe; a.j = j; a.P = P;
    a.yt = W.yt; a.t = W.t; a.tau = W.tau; a.norms = W.norms; a.perm = perm; a.left = W.left;
    a.normref = W.normref;
    a.ctrl = W.ctrl; a.smallest = smallest == 1; a.nopivot = smallest == 2;
    a.semantics = semantics;
    // both kernels start with griddepcontrol.wait, so each may be launched
    // while its predecessor is still running (programmatic dependent launch)
    cudaLaunchAttribute pdl;
    pdl.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL);
    cfg.blockDim = dim3(CT);
    cfg.dynamicSmemBytes = 2 * (size_t)((L + CL - 1) / CL) * 4;
    cfg.stream = st;
    cfg.attrs = &pdl;
    cfg.numAttrs = 1;
    GQ_CHECK_CUDA(cudaLaunchKernelEx(&cfg, qr_step_cluster_kernel, a));
    GQ_TRY(check_launch("qr_step"));
    const int64_t c0 = (semantics == 0) ? pe : j + 1;
    const bool exposes = (semantics == 0) ? (j + 1 < n && pe < n) : (j + 1 < n);
    if (exposes) {
      cfg.gridDim = dim3(gemv_blocks);
      cfg.blockDim = dim3(256);
      cfg.dynamicSmemBytes = 0;
      const float* leftc = W.left;
      const float* ref = semantics == 1 ? W.normref : nullptr;
      GQ_CHECK_CUDA(cudaLaunchKernelEx(&cfg, exposed_row_kernel, (const float*)W.at, m, n, k, c0,
                                       leftc, W.norms, ref, W.ctrl, tol3z));
      GQ_TRY(check_launch("exposed_row"));
    }
  }
  Ctrl h;
  GQ_CHECK_CUDA(cudaMemcpyAsync(&h, W.ctrl, sizeof(Ctrl), cudaMemcpyDeviceToHost, st));
  GQ_CHECK_CUDA(cudaStreamSynchronize(st));
  *width = h.active;
  return GQ_OK;
}

}  // namespace qr
}  // namespace gq

extern "C" {

int64_t gq_qrcp_workspace_size(int64_t m, int64_t n, int panel_size) {
  int P = std::max(1, std::min(panel_size, gq::qr::MAX_P));
  return gq::qr::ws_bytes(m, n, P);
}

int gq_qrcp(float* a, int64_t m, int64_t n, int64_t lda, int panel_size, int pivot_mode,
            int semantics, int32_t* perm, float* v_out, int64_t ldv, float* tau_out,
            int32_t* panel_ends, int* n_panels, void* workspace, int64_t workspace_bytes,
            void* stream) {
  using namespace gq;
  GQ_REQUIRE(a != nullptr && perm != nullptr, "gq_qrcp: NULL a or perm");
  GQ_REQUIRE(m > 0 && n > 0 && lda >= n, "gq_qrcp: bad shape (m=%lld n=%lld lda=%lld)",
             (long long)m, (long long)n, (long long)lda);
  GQ_REQUIRE(panel_size > 0, "panel_size must be positive, got %d", panel_size);
  GQ_REQUIRE(pivot_mode >= 0 && pivot_mode <= 2,
             "gq_qrcp: pivot_mode must be 0 (largest), 1 (smallest) or 2 (none)");
  GQ_REQUIRE(semantics == 0 || semantics == 1, "gq_qrcp: semantics must be 0 or 1");
  GQ_REQUIRE(m * 8 <= 200 * 1024, "gq_qrcp: m=%lld exceeds the step kernel's shared memory", (long long)m);
  GQ_REQUIRE(n < (1ll << 31) && m < (1ll << 31), "gq_qrcp: dimension too large");
  const int64_t limit = std::min(m, n);
  // A panel wider than the matrix is one panel.  The reference semantics depend
  // on the panel width and honour it (up to MAX_P); the intended factorization
  // is independent of it and always runs 64-wide panels.
  int P = (int)std::min<int64_t>(panel_size, limit);
  if (semantics == 1) P = std::min(P, qr::INTENDED_P);
  GQ_REQUIRE(P <= qr::MAX_P, "gq_qrcp: panel_size %d > %d with min(m, n) = %lld is not supported",
             panel_size, qr::MAX_P, (long long)limit);
  GQ_REQUIRE(workspace_bytes >= gq_qrcp_workspace_size(m, n, P), "gq_qrcp: workspace too small");
  GQ_REQUIRE(v_out == nullptr || ldv >= limit, "gq_qrcp: ldv too small");
  cudaStream_t st = as_stream(stream);
  qr::Work W = qr::carve(workspace, m, n, P);
  dim3 tb(32, 8);
  qr::transpose_kernel<<<dim3((unsigned)ceil_div(n, 32), (unsigned)ceil_div(m, 32)), tb, 0, st>>>(
      a, m, n, lda, W.at, m);
  GQ_TRY(check_launch("transpose_in"));
  {
    std::vector<int32_t> iota(n);
    for (int64_t i = 0; i < n; ++i) iota[i] = (int32_t)i;
    GQ_CHECK_CUDA(cudaMemcpyAsync(perm, iota.data(), n * 4, cudaMemcpyHostToDevice, st));
    GQ_CHECK_CUDA(cudaStreamSynchronize(st));
  }
  if (v_out) GQ_CHECK_CUDA(cudaMemset2DAsync(v_out, ldv * 4, 0, limit * 4, m, st));
  if (tau_out) GQ_CHECK_CUDA(cudaMemsetAsync(tau_out, 0, limit * 4, st));
  GQ_TRY(qr::norms_from(W, m, n, 0, true, st));
  int np = 0;
  for (int64_t k = 0; k < limit;) {
    int width = 0;
    GQ_TRY(qr::factor_panel(W, m, n, k, P, pivot_mode, semantics, perm, st, &width));
    const int64_t pe_real = k + width;
    if (panel_ends) panel_ends[np] = (int32_t)pe_real;
    ++np;
    if (v_out && width > 0) {
      qr::store_reflectors_kernel<<<dim3((unsigned)std::min<int64_t>(ceil_div(m, 256), 64),
                                         (unsigned)width), 256, 0, st>>>(W.yt, m, k, width, v_out,
                                                                          ldv, W.tau, tau_out);
      GQ_TRY(check_launch("store_reflectors"));
    }
    GQ_TRY(qr::apply_panel(W, m, n, k, width, P, pe_real, st));
    GQ_TRY(qr::norms_from(W, m, n, pe_real, true, st));
    if (semantics == 0) {
      k += P;  // the reference's driver steps by panel_size regardless (:1665)
    } else {
      if (width == 0) break;  // no mass left ("smallest")
      k = pe_real;
    }
  }
  if (n_panels) *n_panels = np;
  qr::transpose_kernel<<<dim3((unsigned)ceil_div(m, 32), (unsigned)ceil_div(n, 32)), tb, 0, st>>>(
      W.at, n, m, m, a, lda);
  GQ_TRY(check_launch("transpose_out"));
  return GQ_OK;
}

int gq_qr_factor_panel(float* a, int64_t m, int64_t n, int64_t lda, int32_t* perm, float* norms,
                       int64_t k, int panel_size, int pivot_mode, int semantics, float* y_out,
                       float* tau_out, float* t_out, int* panel_end_out, void* workspace,
                       int64_t workspace_bytes, void* stream) {
  using namespace gq;
  GQ_REQUIRE(a && perm && norms && y_out && tau_out && t_out && panel_end_out,
             "gq_qr_factor_panel: NULL argument");
  GQ_REQUIRE(m > 0 && n > 0 && lda >= n, "gq_qr_factor_panel: bad shape");
  const int64_t limit = std::min(m, n);
  GQ_REQUIRE(panel_size > 0, "panel_size must be positive, got %d", panel_size);
  GQ_REQUIRE(k >= 0 && k < limit, "k must be in [0, %lld), got %lld", (long long)limit, (long long)k);
  const int P = (int)std::min<int64_t>(panel_size, limit - k);
  GQ_REQUIRE(P <= qr::MAX_P, "gq_qr_factor_panel: panel width above %d is not supported", qr::MAX_P);
  GQ_REQUIRE(pivot_mode == 0 || pivot_mode == 1, "gq_qr_factor_panel: bad pivot_mode");
  GQ_REQUIRE(semantics == 0 || semantics == 1, "gq_qr_factor_panel: bad semantics");
  GQ_REQUIRE(m * 8 <= 200 * 1024, "gq_qr_factor_panel: m too large");
  GQ_REQUIRE(workspace_bytes >= gq_qrcp_workspace_size(m, n, P), "gq_qr_factor_panel: workspace too small");
  cudaStream_t st = as_stream(stream);
  qr::Work W = qr::carve(workspace, m, n, P);
  dim3 tb(32, 8);
  qr::transpose_kernel<<<dim3((unsigned)ceil_div(n, 32), (unsigned)ceil_div(m, 32)), tb, 0, st>>>(
      a, m, n, lda, W.at, m);
  GQ_TRY(check_launch("transpose_in"));
  GQ_CHECK_CUDA(cudaMemcpyAsync(W.norms, norms, n * 4, cudaMemcpyDeviceToDevice, st));
  GQ_CHECK_CUDA(cudaMemcpyAsync(W.normref, norms, n * 4, cudaMemcpyDeviceToDevice, st));
  int width = 0;
  GQ_TRY(qr::factor_panel(W, m, n, k, P, pivot_mode, semantics, perm, st, &width));
  *panel_end_out = (int)(k + width);
  const int64_t L = m - k;
  // y_out [L, P] (panel-local rows), t_out [P, P], tau_out [P]
  qr::transpose_kernel<<<dim3((unsigned)ceil_div(L, 32), (unsigned)ceil_div(P, 32)), tb, 0, st>>>(
      W.yt, P, L, L, y_out, P);
  GQ_TRY(check_launch("transpose_y"));
  GQ_CHECK_CUDA(cudaMemcpyAsync(t_out, W.t, (size_t)P * P * 4, cudaMemcpyDeviceToDevice, st));
  GQ_CHECK_CUDA(cudaMemcpyAsync(tau_out, W.tau, (size_t)P * 4, cudaMemcpyDeviceToDevice, st));
  GQ_CHECK_CUDA(cudaMemcpyAsync(norms, W.norms, n * 4, cudaMemcpyDeviceToDevice, st));
  qr::transpose_kernel<<<dim3((unsigned)ceil_div(m, 32), (unsigned)ceil_div(n, 32)), tb, 0, st>>>(
      W.at, n, m, m, a, lda);
  return check_launch("transpose_out");
}

int gq_qr_apply_panel(float* b, int64_t rows, int64_t cols, int64_t ldb, const float* y,
                      int64_t ldy, const float* t, int64_t ldt, int width, float* scratch,
                      void* stream) {
  using namespace gq;
  GQ_REQUIRE(rows >= 0 && cols >= 0 && width >= 0, "gq_qr_apply_panel: negative size");
  GQ_REQUIRE(ldb >= cols && ldy >= width && ldt >= width, "gq_qr_apply_panel: bad leading dims");
  if (rows == 0 || cols == 0 || width == 0) return GQ_OK;
  GQ_REQUIRE(b && y && t && scratch, "gq_qr_apply_panel: NULL argument");
  cudaStream_t st = as_stream(stream);
  float* w1 = scratch;                   // width x cols
  float* w2 = scratch + (int64_t)width * cols;
  GQ_TRY(sgemm(1, 0, width, cols, rows, 1.f, y, ldy, b, ldb, 0.f, w1, cols, 0, st));
  GQ_TRY(sgemm(1, 0, width, cols, width, 1.f, t, ldt, w1, cols, 0.f, w2, cols, 0, st));
  return sgemm(0, 0, rows, cols, width, -1.f, y, ldy, w2, cols, 1.f, b, ldb, 0, st);
}

}  // extern "C"
