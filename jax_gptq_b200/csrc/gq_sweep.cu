// GPTQ column sweep with lazy batch updates (Frantar et al., 2022) -- the
// computation gptq_ref.py:136-155 stands in for.  With U = I every error
// update is an exact zero and the result is gptq_forward_step bit for bit.
//
// Data layout (workspace): wp [m, ldp] float32 -- the working weights in
// permuted column order (ldp = n rounded up to 4), overwritten block by block
// with the dequantized values; cp [m, ldp] uint8 -- codes in permuted order;
// err [m, 128] float32 -- the scaled errors of the current block.
//
// Per 128-column block:
//   1. sweep_block_kernel: a warp owns 4 rows; lane l holds columns 4l..4l+3
//      of each in registers; the block of U lives in shared memory.  For each
//      column i, lane r < 4 gathers row r's current value, quantizes it once,
//      writes the code / dequantized value / error and broadcasts the error
//      (w - dq) / U_ii, which every lane applies to its columns > i.
//   2. wp[:, b1:] -= err @ U[b0:b1, b1:]  (fp32 GEMM).
// Finally codes/dequant are scattered back to original column order.
#include "gq_common.cuh"
#include "gq_quant.cuh"

namespace gq {

int sgemm(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
          const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int uplo, cudaStream_t st);
int check_quant_args(const char* who, int64_t m, int64_t n, int w_bits, int group_size, int sym);

constexpr int SW_BLOCK = 128;
constexpr int SW_ROWS = 4;        // rows per warp (lane r < 4 quantizes row r)
constexpr int SW_WARPS = 4;       // warps per CTA
constexpr int SW_ROWS_CTA = SW_ROWS * SW_WARPS;

inline int64_t round4(int64_t n) { return (n + 3) & ~int64_t(3); }

// wp[r][j] = src[r][perm[j]]   (or a plain copy of start, already permuted)
__global__ void gather_rows_kernel(const float* __restrict__ w, int64_t n, int64_t ldw,
                                   const int32_t* __restrict__ perm, float* __restrict__ wp,
                                   int64_t ldp) {
  extern __shared__ __align__(16) float srow[];
  const int64_t r = blockIdx.x;
  const float* wr = w + r * ldw;
  for (int64_t c = threadIdx.x; c < n; c += blockDim.x) srow[c] = wr[c];
  __syncthreads();
  float* out = wp + r * ldp;
  for (int64_t j = threadIdx.x; j < ldp; j += blockDim.x)
    out[j] = (j < n) ? srow[perm ? perm[j] : j] : 0.f;
}

// Group parameters for a group that spans more than one block (g % 128 == 0):
// computed from the current permuted weights wp[:, c0:c0+g] at the group start.
__global__ void group_params_kernel(const float* __restrict__ wp, int64_t m, int64_t ldp,
                                    int64_t c0, int g, QParams qp, int sym,
                                    float* __restrict__ gscale, float* __restrict__ gzero) {
  const int lane = threadIdx.x & 31;
  const int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= m) return;
  const float* row = wp + r * ldp + c0;
  float mn = INFINITY, mx = -INFINITY, ma = 0.f;
  for (int e = lane; e < g; e += 32) {
    float v = row[e];
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
    gscale[r] = s;
    gzero[r] = z;
  }
}

struct SweepArgs {
  float* wp;            // [m, ldp]
  uint8_t* cp;          // [m, ldp]
  float* err;           // [m, 128]
  const float* u;       // [n, ldu]
  int64_t m, n, ldp, ldu;
  int64_t b0;           // first column of this block
  int bw;               // block width (<= 128)
  int g;                // group size
  int n_groups;
  QParams qp;
  int sym;
  int noprop_cols;
  const float* group0_scale;  // nullable
  const float* group0_zero;
  const float* big_scale;     // [m] params of the current group when g > 128
  const float* big_zero;
  float* scales;              // [m, n_groups] nullable
  float* zeros;
};

__global__ void __launch_bounds__(SW_WARPS * 32)
sweep_block_kernel(SweepArgs a) {
  extern __shared__ __align__(16) float sweep_smem[];
  float (*us)[SW_BLOCK] = reinterpret_cast<float (*)[SW_BLOCK]>(sweep_smem);
  float* udinv = sweep_smem + SW_BLOCK * SW_BLOCK;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int bw = a.bw;
  // U block into shared memory (zero beyond the block width)
  for (int e = threadIdx.x; e < SW_BLOCK * SW_BLOCK; e += blockDim.x) {
    int r = e >> 7, c = e & 127;
    us[r][c] = (r < bw && c < bw) ? a.u[(a.b0 + r) * a.ldu + a.b0 + c] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < SW_BLOCK; i += blockDim.x) udinv[i] = (i < bw) ? 1.f / us[i][i] : 0.f;
  __syncthreads();

  // Lane l holds columns 4l..4l+3 of the warp's SW_ROWS rows; lane r < SW_ROWS
  // additionally "owns" row r: it quantizes that row's current column and
  // writes its outputs, so every quantization is computed exactly once.
  const int64_t row_base = (int64_t)blockIdx.x * SW_ROWS_CTA + warp * SW_ROWS;
  const bool row_lane = lane < SW_ROWS;
  const int64_t my_row = row_base + lane;
  const bool my_valid = row_lane && my_row < a.m;
  float w[SW_ROWS][4];
#pragma unroll
  for (int r = 0; r < SW_ROWS; ++r) {
    const int64_t row = row_base + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (row < a.m && 4 * lane < bw)
      v = *reinterpret_cast<const float4*>(a.wp + row * a.ldp + a.b0 + 4 * lane);
    w[r][0] = v.x; w[r][1] = v.y; w[r][2] = v.z; w[r][3] = v.w;
  }
  float my_scale = 1.f, my_zero = 0.f;
  if (a.g > SW_BLOCK && my_valid) {
    my_scale = a.big_scale[my_row];
    my_zero = a.big_zero[my_row];
  }
  float* wrow = my_valid ? a.wp + my_row * a.ldp + a.b0 : nullptr;
  uint8_t* crow = my_valid ? a.cp + my_row * a.ldp + a.b0 : nullptr;
  float* erow = my_valid ? a.err + my_row * SW_BLOCK : nullptr;
  const int seg = (a.g <= SW_BLOCK) ? (a.g >> 2) : 32;  // lanes per group inside a block

  for (int i4 = 0; i4 < bw; i4 += 4) {
    const int owner = i4 >> 2;
#pragma unroll
    for (int sub = 0; sub < 4; ++sub) {
      const int i = i4 + sub;
      if (i >= bw) break;
      // group parameters at the group's first column, from the current values
      // (g divides 128 here and blocks start on group boundaries, so the test
      // on the block-local index is a mask)
      if (a.g <= SW_BLOCK && (i & (a.g - 1)) == 0) {
        const int64_t gi = (a.b0 + i) / a.g;
#pragma unroll
        for (int r = 0; r < SW_ROWS; ++r) {
          float mn = INFINITY, mx = -INFINITY, ma = 0.f;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            if (4 * lane + t < bw) {
              mn = fminf(mn, w[r][t]);
              mx = fmaxf(mx, w[r][t]);
              ma = fmaxf(ma, fabsf(w[r][t]));
            }
          }
          for (int o = 1; o < seg; o <<= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, o));
          }
          mn = __shfl_sync(0xffffffffu, mn, owner);
          mx = __shfl_sync(0xffffffffu, mx, owner);
          ma = __shfl_sync(0xffffffffu, ma, owner);
          if (lane == r) {
            float s, z;
            if (gi == 0 && a.group0_scale != nullptr) {
              s = my_valid ? a.group0_scale[my_row] : 1.f;
              z = my_valid ? a.group0_zero[my_row] : 0.f;
            } else if (a.sym) {
              group_scale_zero(-ma, ma, a.qp, a.sym, s, z);
            } else {
              group_scale_zero(mn, mx, a.qp, a.sym, s, z);
            }
            my_scale = s;
            my_zero = z;
            if (my_valid && a.scales) {
              a.scales[my_row * a.n_groups + gi] = s;
              a.zeros[my_row * a.n_groups + gi] = z;
            }
          }
        }
      }
      // gather column i of each row into its row lane
      float mine = 0.f;
#pragma unroll
      for (int r = 0; r < SW_ROWS; ++r) {
        const float v = __shfl_sync(0xffffffffu, w[r][sub], owner);
        if (lane == r) mine = v;
      }
      const bool prop = a.b0 + i >= a.noprop_cols;
      float dq;
      const float q = quantize_one(mine, my_scale, my_zero, a.qp, dq);
      const float my_err = prop ? __fmul_rn(__fsub_rn(mine, dq), udinv[i]) : 0.f;
      if (my_valid) {
        wrow[i] = dq;
        crow[i] = (uint8_t)(int)(q - a.qp.qmin);
        erow[i] = my_err;
      }
      const float4 urow = *reinterpret_cast<const float4*>(&us[i][4 * lane]);
      const float uv[4] = {urow.x, urow.y, urow.z, urow.w};
#pragma unroll
      for (int r = 0; r < SW_ROWS; ++r) {
        const float err = __shfl_sync(0xffffffffu, my_err, r);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          if (4 * lane + t > i) w[r][t] = fmaf(-err, uv[t], w[r][t]);
        }
      }
    }
  }
}

// dequant[r][perm[j]] = wp[r][j], codes likewise (scatter through shared memory).
__global__ void unpermute_rows_kernel(const float* __restrict__ wp, const uint8_t* __restrict__ cp,
                                      int64_t n, int64_t ldp, const int32_t* __restrict__ perm,
                                      float* __restrict__ dequant, uint8_t* __restrict__ codes) {
  extern __shared__ __align__(16) unsigned char sm[];
  float* sval = reinterpret_cast<float*>(sm);
  uint8_t* scode = reinterpret_cast<uint8_t*>(sval + n);
  const int64_t r = blockIdx.x;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) {
    int64_t c = perm ? perm[j] : j;
    sval[c] = wp[r * ldp + j];
    scode[c] = cp[r * ldp + j];
  }
  __syncthreads();
  if (dequant)
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) dequant[r * n + c] = sval[c];
  if (codes)
    for (int64_t c = threadIdx.x; c < n; c += blockDim.x) codes[r * n + c] = scode[c];
}

__global__ void g_idx_kernel(const int32_t* __restrict__ perm, int64_t n, int g, int32_t* g_idx) {
  int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (j < n) g_idx[perm ? perm[j] : j] = (int32_t)(j / g);
}

// Byte offset of the transposed U band (after wp, cp, err, bscale, bzero).
inline int64_t sweep_ubt_offset(int64_t m, int64_t n) {
  int64_t ldp = round4(n);
  int64_t off = m * ldp * 4 + ((m * ldp + 15) & ~int64_t(15)) + m * SW_BLOCK * 4 + 2 * m * 4;
  return (off + 255) & ~int64_t(255);
}

int64_t sweep_ws_bytes(int64_t m, int64_t n) {
  return sweep_ubt_offset(m, n) + n * SW_BLOCK * 4 + 256;
}

int transpose2d(const float* src, int64_t rows, int64_t cols, int64_t lds, float* dst, int64_t ldd,
                cudaStream_t st);

}  // namespace gq

extern "C" {

int64_t gq_gptq_sweep_workspace_size(int64_t m, int64_t n) { return gq::sweep_ws_bytes(m, n); }

int gq_gptq_sweep(const float* w, int64_t m, int64_t n, int64_t ldw, const float* start,
                  const float* u, int64_t ldu, const int32_t* perm, int w_bits, int group_size,
                  int sym, int block, const float* group0_scale, const float* group0_zero,
                  int noprop_cols, float* dequant, uint8_t* codes, float* scales, float* zeros,
                  int32_t* g_idx, void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace gq;
  GQ_TRY(check_quant_args("gq_gptq_sweep", m, n, w_bits, group_size, sym));
  GQ_REQUIRE(block == SW_BLOCK, "gq_gptq_sweep: block must be %d", SW_BLOCK);
  GQ_REQUIRE((SW_BLOCK % group_size == 0 && group_size >= 4) || group_size % SW_BLOCK == 0,
             "gq_gptq_sweep: group_size %d must divide 128 (>= 4) or be a multiple of 128",
             group_size);
  GQ_REQUIRE(u != nullptr && ldu >= n, "gq_gptq_sweep: bad u");
  GQ_REQUIRE(w != nullptr && ldw >= n, "gq_gptq_sweep: bad w");
  GQ_REQUIRE((group0_scale == nullptr) == (group0_zero == nullptr),
             "gq_gptq_sweep: group0_scale and group0_zero must both be given or both NULL");
  GQ_REQUIRE((scales == nullptr) == (zeros == nullptr),
             "gq_gptq_sweep: scales and zeros must both be given or both NULL");
  GQ_REQUIRE(workspace_bytes >= sweep_ws_bytes(m, n), "gq_gptq_sweep: workspace too small");
  GQ_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
             "gq_gptq_sweep: workspace must be 256-byte aligned");
  GQ_REQUIRE(n * 5 + 64 <= 220 * 1024, "gq_gptq_sweep: n=%lld exceeds the row buffer",
             (long long)n);
  if (m == 0 || n == 0) return GQ_OK;
  cudaStream_t st = as_stream(stream);
  const int64_t ldp = round4(n);
  char* ws = reinterpret_cast<char*>(workspace);
  float* wp = reinterpret_cast<float*>(ws);
  uint8_t* cp = reinterpret_cast<uint8_t*>(ws + m * ldp * 4);
  float* err = reinterpret_cast<float*>(ws + m * ldp * 4 + ((m * ldp + 15) & ~int64_t(15)));
  float* bscale = err + m * SW_BLOCK;
  float* bzero = bscale + m;
  float* ubt = reinterpret_cast<float*>(ws + sweep_ubt_offset(m, n));  // [n, 128]

  if (start) {
    GQ_CHECK_CUDA(cudaMemcpy2DAsync(wp, ldp * 4, start, n * 4, n * 4, m, cudaMemcpyDeviceToDevice, st));
  } else {
    size_t smem = (size_t)n * 4;
    GQ_CHECK_CUDA(cudaFuncSetAttribute(gather_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
    gather_rows_kernel<<<(unsigned)m, 256, smem, st>>>(w, n, ldw, perm, wp, ldp);
    GQ_TRY(check_launch("gather_rows"));
  }

  SweepArgs a;
  a.wp = wp; a.cp = cp; a.err = err; a.u = u;
  a.m = m; a.n = n; a.ldp = ldp; a.ldu = ldu;
  a.g = group_size; a.n_groups = (int)(n / group_size);
  a.qp = make_qparams(w_bits, sym); a.sym = sym;
  a.noprop_cols = noprop_cols;
  a.group0_scale = group0_scale; a.group0_zero = group0_zero;
  a.big_scale = bscale; a.big_zero = bzero;
  a.scales = scales; a.zeros = zeros;
  const unsigned grid = (unsigned)ceil_div(m, SW_ROWS_CTA);
  const size_t sweep_smem_bytes = (SW_BLOCK * SW_BLOCK + SW_BLOCK) * sizeof(float);
  GQ_CHECK_CUDA(cudaFuncSetAttribute(sweep_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)sweep_smem_bytes));
  for (int64_t b0 = 0; b0 < n; b0 += SW_BLOCK) {
    const int bw = (int)std::min<int64_t>(SW_BLOCK, n - b0);
    if (group_size > SW_BLOCK && b0 % group_size == 0) {
      const int64_t gi = b0 / group_size;
      if (gi == 0 && group0_scale) {
        GQ_CHECK_CUDA(cudaMemcpyAsync(bscale, group0_scale, m * 4, cudaMemcpyDeviceToDevice, st));
        GQ_CHECK_CUDA(cudaMemcpyAsync(bzero, group0_zero, m * 4, cudaMemcpyDeviceToDevice, st));
      } else {
        group_params_kernel<<<(unsigned)ceil_div(m, 8), 256, 0, st>>>(wp, m, ldp, b0, group_size,
                                                                      a.qp, sym, bscale, bzero);
        GQ_TRY(check_launch("group_params"));
      }
      if (scales) {
        GQ_CHECK_CUDA(cudaMemcpy2DAsync(scales + gi, a.n_groups * 4, bscale, 4, 4, m,
                                        cudaMemcpyDeviceToDevice, st));
        GQ_CHECK_CUDA(cudaMemcpy2DAsync(zeros + gi, a.n_groups * 4, bzero, 4, 4, m,
                                        cudaMemcpyDeviceToDevice, st));
      }
    }
    a.b0 = b0;
    a.bw = bw;
    sweep_block_kernel<<<grid, SW_WARPS * 32, sweep_smem_bytes, st>>>(a);
    GQ_TRY(check_launch("sweep_block"));
    const int64_t b1 = b0 + bw;
    if (b1 < n) {
      // wp[:, b1:] -= err @ U[b0:b1, b1:], with the U band transposed so that
      // both GEMM operands are K-major (tensor-core path)
      GQ_TRY(transpose2d(u + b0 * ldu + b1, bw, n - b1, ldu, ubt, SW_BLOCK, st));
      GQ_TRY(sgemm(0, 1, m, n - b1, bw, -1.f, err, SW_BLOCK, ubt, SW_BLOCK, 1.f, wp + b1, ldp, 0,
                   st));
    }
  }
  if (dequant || codes) {
    size_t smem = (size_t)n * 5 + 16;
    GQ_CHECK_CUDA(cudaFuncSetAttribute(unpermute_rows_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    unpermute_rows_kernel<<<(unsigned)m, 256, smem, st>>>(wp, cp, n, ldp, perm, dequant, codes);
    GQ_TRY(check_launch("unpermute_rows"));
  }
  if (g_idx) {
    g_idx_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(perm, n, group_size, g_idx);
    GQ_TRY(check_launch("g_idx"));
  }
  return GQ_OK;
}

}  // extern "C"
