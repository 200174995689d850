// Qronos single-layer update on the device (the computation
// qronos_ref.py:7-25 stands in for).  With Xt the quantized-model and X the
// float activations, h = Xt^T Xt (damped: hd, in permuted coordinates),
// g = X^T Xt and U = chol(hd^-1, upper):
//   rhs   = W_orig[:, p] @ g[p][:, p]          (row r: (g^T w_orig)_perm)
//   v1    = (rhs[:, 0] - W[:, p][:, 1:] @ hd[0, 1:]) / hd[0, 0]
//   q1    = Q(v1) with group-0 parameters from W[:, p][:, :group]
//   b     = rhs[:, 1:] - dq1 * hd[0, 1:]
//   W1    = b @ U2^T @ U2     (U2 = U[1:, 1:], so U2^T U2 = hd[1:, 1:]^-1)
// then the GPTQ sweep runs on [v1 | W1] with column 0 fixed (no error
// propagation) and group 0's parameters preset.
#include "gq_common.cuh"
#include "gq_quant.cuh"

namespace gq {

int sgemm(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
          const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int uplo, cudaStream_t st);
int sgemm_tri(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A,
              int64_t lda, const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int tri,
              cudaStream_t st);
int transpose2d(const float* src, int64_t rows, int64_t cols, int64_t lds, float* dst, int64_t ldd,
                cudaStream_t st);
int rtn_launch(const float* w, int64_t m, int64_t n, int64_t ldw, const int32_t* perm, int w_bits,
               int group_size, int sym, float* dequant, uint8_t* codes, float* scales, float* zeros,
               cudaStream_t st);
int check_quant_args(const char* who, int64_t m, int64_t n, int w_bits, int group_size, int sym);
int64_t sweep_ws_bytes(int64_t m, int64_t n);

// out[r][j] = a[r][perm[j]]   (rows of length n, ld n)
__global__ void permute_cols_kernel(const float* __restrict__ a, int64_t n,
                                    const int32_t* __restrict__ perm, float* __restrict__ out) {
  const int64_t r = blockIdx.y;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x)
    out[r * n + j] = a[r * n + (perm ? perm[j] : j)];
}

// out[i][j] = a[perm[i]][perm[j]]
__global__ void permute_square_kernel(const float* __restrict__ a, int64_t n,
                                      const int32_t* __restrict__ perm, float* __restrict__ out) {
  const int64_t i = blockIdx.y;
  const int64_t pi = perm ? perm[i] : i;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x)
    out[i * n + j] = a[pi * n + (perm ? perm[j] : j)];
}

// up[i][j] = u[i][j] with row 0 and column 0 cleared, so that
// up^T up = [[0, 0], [0, U2^T U2]] for U2 = u[1:, 1:]
__global__ void pad_u_kernel(const float* __restrict__ u, int64_t n, float* __restrict__ up) {
  const int64_t i = blockIdx.y;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x)
    up[i * n + j] = (i == 0 || j == 0) ? 0.f : u[i * n + j];
}

// t[r] = sum_{j >= 1} a[r][j] * hrow[j]   (one warp per row)
__global__ void row_dot_tail_kernel(const float* __restrict__ a, int64_t m, int64_t n,
                                    const float* __restrict__ hrow, float* __restrict__ t) {
  const int lane = threadIdx.x & 31;
  const int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= m) return;
  const float* ar = a + r * n;
  float s = 0.f;
  for (int64_t j = 1 + lane; j < n; j += 32) s = fmaf(ar[j], hrow[j], s);
  s = warp_sum(s);
  if (lane == 0) t[r] = s;
}

// v1 = (rhs0 - t) / hd00;  dq1 = Q(v1) with group-0 parameters
__global__ void qronos_first_col_kernel(const float* __restrict__ rhs, const float* __restrict__ t,
                                        const float* __restrict__ hd, int64_t m, int64_t n,
                                        const float* __restrict__ s0, const float* __restrict__ z0,
                                        QParams qp, float* __restrict__ v1_out,
                                        float* __restrict__ dq1) {
  int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= m) return;
  float v1 = (rhs[r * n] - t[r]) / hd[0];
  float dq;
  quantize_one(v1, s0[r], z0[r], qp, dq);
  v1_out[r] = v1;
  dq1[r] = dq;
}

// b[r][j] = rhs[r][j] - dq1[r] * hd[0][j] for j >= 1, b[r][0] = 0  (in place)
__global__ void qronos_rank1_kernel(float* __restrict__ rhs, int64_t n,
                                    const float* __restrict__ dq1, const float* __restrict__ hrow) {
  const int64_t r = blockIdx.y;
  const float d = dq1[r];
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x)
    rhs[r * n + j] = (j == 0) ? 0.f : __fsub_rn(rhs[r * n + j], __fmul_rn(d, hrow[j]));
}

__global__ void set_col0_kernel(float* __restrict__ a, int64_t m, int64_t n,
                                const float* __restrict__ v) {
  int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r < m) a[r * n] = v[r];
}

// workspace floats before the sweep's own workspace: g^T, permuted (n*n);
// U padded and its transpose (2*n*n); three m*n buffers; four m-vectors
int64_t qronos_head_floats(int64_t m, int64_t n) { return 3 * n * n + 3 * m * n + 4 * m + 64; }

int64_t qronos_ws_bytes(int64_t m, int64_t n) {
  int64_t a = (qronos_head_floats(m, n) * 4 + 255) & ~int64_t(255);
  return a + sweep_ws_bytes(m, n);
}

}  // namespace gq

extern "C" {

int64_t gq_qronos_workspace_size(int64_t m, int64_t n) { return gq::qronos_ws_bytes(m, n); }

int gq_gptq_sweep(const float* w, int64_t m, int64_t n, int64_t ldw, const float* start,
                  const float* u, int64_t ldu, const int32_t* perm, int w_bits, int group_size,
                  int sym, int block, const float* group0_scale, const float* group0_zero,
                  int noprop_cols, float* dequant, uint8_t* codes, float* scales, float* zeros,
                  int32_t* g_idx, void* workspace, int64_t workspace_bytes, void* stream);

int gq_qronos(const float* w, const float* w_orig, int64_t m, int64_t n, const float* hd,
              const float* u, const float* g, const int32_t* perm, int w_bits, int group_size,
              int sym, int block, float* dequant, uint8_t* codes, float* scales, float* zeros,
              int32_t* g_idx, void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace gq;
  GQ_TRY(check_quant_args("gq_qronos", m, n, w_bits, group_size, sym));
  GQ_REQUIRE(w && w_orig && hd && u && g, "gq_qronos: NULL input");
  GQ_REQUIRE(n >= 2, "gq_qronos: needs at least two columns");
  GQ_REQUIRE(workspace_bytes >= qronos_ws_bytes(m, n), "gq_qronos: workspace too small");
  GQ_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
             "gq_qronos: workspace must be 256-byte aligned");
  if (m == 0) return GQ_OK;
  cudaStream_t st = as_stream(stream);
  float* ws = reinterpret_cast<float*>(workspace);
  float* gpt = ws;                // n*n: (g_p)^T = (g^T)_p; first g^T
  float* up = gpt + n * n;        // n*n: U with row/column 0 cleared
  float* upt = up + n * n;        // n*n: up^T
  float* bufA = upt + n * n;      // m*n: W[:, p], later b up^T
  float* bufB = bufA + m * n;     // m*n: W_orig[:, p], later the sweep start
  float* rhs = bufB + m * n;      // m*n: rhs, then b (column 0 cleared)
  float* s0 = rhs + m * n;        // m
  float* z0 = s0 + m;             // m
  float* tv = z0 + m;             // m: t, then v1
  float* dq1 = tv + m;            // m
  int64_t head = (qronos_head_floats(m, n) * 4 + 255) & ~int64_t(255);
  void* sweep_ws = reinterpret_cast<char*>(workspace) + head;
  int64_t sweep_bytes = workspace_bytes - head;
  const unsigned gx = (unsigned)std::min<int64_t>(ceil_div(n, 256), 64);

  // (g_p)^T[i][j] = g[p[j]][p[i]] = (g^T)[p[i]][p[j]]: transpose, then permute
  GQ_TRY(transpose2d(g, n, n, n, upt, n, st));
  permute_square_kernel<<<dim3(gx, (unsigned)n), 256, 0, st>>>(upt, n, perm, gpt);
  GQ_TRY(check_launch("permute_square"));
  pad_u_kernel<<<dim3(gx, (unsigned)n), 256, 0, st>>>(u, n, up);
  GQ_TRY(check_launch("pad_u"));
  GQ_TRY(transpose2d(up, n, n, n, upt, n, st));
  permute_cols_kernel<<<dim3(gx, (unsigned)m), 256, 0, st>>>(w, n, perm, bufA);
  permute_cols_kernel<<<dim3(gx, (unsigned)m), 256, 0, st>>>(w_orig, n, perm, bufB);
  GQ_TRY(check_launch("permute_cols"));
  // rhs = W_orig[:, p] @ g_p
  GQ_TRY(sgemm(0, 1, m, n, n, 1.f, bufB, n, gpt, n, 0.f, rhs, n, 0, st));
  // group-0 parameters from the starting weights
  GQ_TRY(rtn_launch(bufA, m, group_size, n, nullptr, w_bits, group_size, sym, nullptr, nullptr, s0,
                    z0, st));
  // t = W[:, p][:, 1:] @ hd[0, 1:];  v1, dq1
  row_dot_tail_kernel<<<(unsigned)ceil_div(m, 8), 256, 0, st>>>(bufA, m, n, hd, tv);
  GQ_TRY(check_launch("row_dot_tail"));
  qronos_first_col_kernel<<<(unsigned)ceil_div(m, 256), 256, 0, st>>>(
      rhs, tv, hd, m, n, s0, z0, make_qparams(w_bits, sym), tv, dq1);
  GQ_TRY(check_launch("qronos_first_col"));
  // b = rhs[:, 1:] - dq1 hd[0, 1:]  (column 0 cleared)
  qronos_rank1_kernel<<<dim3(gx, (unsigned)m), 256, 0, st>>>(rhs, n, dq1, hd);
  GQ_TRY(check_launch("qronos_rank1"));
  // W1 = (b U2^T) U2 on padded operands: [0 | W1] = (b_full up^T) up
  GQ_TRY(sgemm_tri(0, 1, m, n, n, 1.f, rhs, n, up, n, 0.f, bufA, n, 4, st));
  GQ_TRY(sgemm_tri(0, 1, m, n, n, 1.f, bufA, n, upt, n, 0.f, bufB, n, 3, st));
  set_col0_kernel<<<(unsigned)ceil_div(m, 256), 256, 0, st>>>(bufB, m, n, tv);
  GQ_TRY(check_launch("set_col0"));
  return gq_gptq_sweep(w, m, n, n, bufB, u, n, perm, w_bits, group_size, sym, block, s0, z0, 1,
                       dequant, codes, scales, zeros, g_idx, sweep_ws, sweep_bytes, stream);
}

}  // extern "C"
