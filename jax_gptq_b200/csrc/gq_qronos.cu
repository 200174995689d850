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

// v1 = (rhs0 - t) / hd00 -> start[:, 0]; dq1 = Q(v1)
__global__ void qronos_first_col_kernel(const float* __restrict__ rhs, const float* __restrict__ t,
                                        const float* __restrict__ hd, int64_t m, int64_t n,
                                        const float* __restrict__ s0, const float* __restrict__ z0,
                                        QParams qp, float* __restrict__ start,
                                        float* __restrict__ dq1) {
  int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= m) return;
  float v1 = (rhs[r * n] - t[r]) / hd[0];
  float dq;
  quantize_one(v1, s0[r], z0[r], qp, dq);
  start[r * n] = v1;
  dq1[r] = dq;
}

int64_t qronos_ws_bytes(int64_t m, int64_t n) {
  int64_t f = n * n + 3 * m * n + 4 * m + 64;
  int64_t a = (f * 4 + 255) & ~int64_t(255);
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
  float* gp = ws;                 // n*n
  float* bufA = gp + n * n;       // m*n: W[:, p], later b U2^T
  float* bufB = bufA + m * n;     // m*n: W_orig[:, p], later the sweep start
  float* rhs = bufB + m * n;      // m*n
  float* s0 = rhs + m * n;        // m
  float* z0 = s0 + m;             // m
  float* tv = z0 + m;             // m
  float* dq1 = tv + m;            // m
  int64_t head = ((n * n + 3 * m * n + 4 * m + 64) * 4 + 255) & ~int64_t(255);
  void* sweep_ws = reinterpret_cast<char*>(workspace) + head;
  int64_t sweep_bytes = workspace_bytes - head;

  dim3 gsq((unsigned)std::min<int64_t>(ceil_div(n, 256), 64), (unsigned)n);
  permute_square_kernel<<<gsq, 256, 0, st>>>(g, n, perm, gp);
  GQ_TRY(check_launch("permute_square"));
  dim3 gcol((unsigned)std::min<int64_t>(ceil_div(n, 256), 64), (unsigned)m);
  permute_cols_kernel<<<gcol, 256, 0, st>>>(w, n, perm, bufA);
  permute_cols_kernel<<<gcol, 256, 0, st>>>(w_orig, n, perm, bufB);
  GQ_TRY(check_launch("permute_cols"));
  // rhs = W_orig[:, p] @ g_p
  GQ_TRY(sgemm(0, 0, m, n, n, 1.f, bufB, n, gp, n, 0.f, rhs, n, 0, st));
  // group-0 parameters from the starting weights
  GQ_TRY(rtn_launch(bufA, m, group_size, n, nullptr, w_bits, group_size, sym, nullptr, nullptr, s0,
                    z0, st));
  // t = W[:, p][:, 1:] @ hd[0, 1:]
  GQ_TRY(sgemm(0, 1, m, 1, n - 1, 1.f, bufA + 1, n, hd + 1, n, 0.f, tv, 1, 0, st));
  qronos_first_col_kernel<<<(unsigned)ceil_div(m, 256), 256, 0, st>>>(
      rhs, tv, hd, m, n, s0, z0, make_qparams(w_bits, sym), bufB, dq1);
  GQ_TRY(check_launch("qronos_first_col"));
  // b = rhs[:, 1:] - dq1 hd[0, 1:]
  GQ_TRY(sgemm(0, 0, m, n - 1, 1, -1.f, dq1, 1, hd + 1, n, 1.f, rhs + 1, n, 0, st));
  // W1 = (b U2^T) U2
  GQ_TRY(sgemm(0, 1, m, n - 1, n - 1, 1.f, rhs + 1, n, u + n + 1, n, 0.f, bufA, n, 0, st));
  GQ_TRY(sgemm(0, 0, m, n - 1, n - 1, 1.f, bufA, n, u + n + 1, n, 0.f, bufB + 1, n, 0, st));
  return gq_gptq_sweep(w, m, n, n, bufB, u, n, perm, w_bits, group_size, sym, block, s0, z0, 1,
                       dequant, codes, scales, zeros, g_idx, sweep_ws, sweep_bytes, stream);
}

}  // extern "C"
