// GPTQ column sweep with lazy batch updates (Frantar et al., 2022) -- the
// computation gptq_ref.py:136-155 stands in for.  With U = I every error
// update is an exact zero and the result is gptq_forward_step bit for bit.
//
// Data layout (workspace): wp [m, ldp] float32 -- the working weights in
// permuted column order (ldp = n rounded up to 4), overwritten block by block
// with the dequantized values; cp [m, ldp] uint8 -- codes in permuted order;
// err [m, 512] float32 -- the scaled errors of the current super-block.
//
// The lazy updates are two-level: blocks of 128 columns inside super-blocks
// of 512.  Per block [b0, b1) of super-block [s0, s1):
//   0. (once per super-block) U[s0:s1, s0:n] is transposed into ubt, so
//      column j of U's super-block rows is one contiguous run of <= 512
//      floats; the band of every block and both GEMMs' U operands are views
//      of it;
//   1. the block's own 128 x 128 band U[b0:b1, b0:b1] is staged in shared
//      memory (cp.async) by the block-step kernel;
//   2. the block step, one lane per weight row: the lane quantizes its row's
//      columns one by one (32-column sub-blocks in registers, the rest of the
//      block in a shared-memory row buffer) and writes codes, dequantized
//      values and scaled errors (w - dq) / U_ii into its 128 columns of err.
//      sweep_rows_kernel runs it on four warps per 32 rows (one for the
//      column chain, three applying finished sub-blocks' errors ahead of it),
//      with 1, 2 or 4 such row groups per CTA sharing one staged band;
//      sweep_rows1_kernel, on one warp, serves grids too large for one wave
//      of those CTAs;
//   3. near update: wp[:, b1:s1] -= err[:, b0-s0:b1-s0] @ U[b0:b1, b1:s1].
// After the super-block, one far update with K = 512:
//   wp[:, s1:] -= err @ U[s0:s1, s1:]   (U[s0:s1, s1:] transposed first).
// The far update is most of the work; at K = 512 it moves a quarter of the
// weight traffic of four K = 128 updates and keeps the tensor cores busier.
// A group wider than a block must not start inside a super-block and end
// past it (its parameters are taken from the columns at its start, before
// the far update); other group sizes fall back to 128-column super-blocks.
// Finally codes/dequant are scattered back to original column order.
#include <atomic>

#include "gq_common.cuh"
#include "gq_quant.cuh"

namespace gq {

int sgemm(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
          const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int uplo, cudaStream_t st);
int check_quant_args(const char* who, int64_t m, int64_t n, int w_bits, int group_size, int sym);

constexpr int SW_BLOCK = 128;
constexpr int SW_SUPER = 512;  // columns per super-block (far updates)
constexpr int SW_SUB = 32;   // columns of a register-resident sub-block
constexpr int SW_WP = 33;    // pitch of the row buffer (lane-private columns, conflict-free)
constexpr int SW_TP = 36;    // pitch of the sub-block U tile (16-byte rows for broadcast reads)

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
  float* err;           // [m, ld_err]: this block's scaled errors
  int64_t ld_err;
  const float* ubt;     // band: ubt[j * ldub + i] = U[b0 + i][b0 + j]
  int64_t ldub;
  int64_t m, n, ldp;
  int64_t b0;           // first column of this block
  int bw;               // block width (<= 128)
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

// Scale / zero of lane's row from its running min, max and max |w|; group 0
// may take caller-supplied parameters.
__device__ __forceinline__ void sweep_group_params(const SweepArgs& a, int64_t row, bool valid,
                                                   int64_t gi, float mn, float mx, float ma,
                                                   float& scale, float& zero) {
  if (gi == 0 && a.group0_scale != nullptr) {
    scale = valid ? a.group0_scale[row] : 1.f;
    zero = valid ? a.group0_zero[row] : 0.f;
  } else if (a.sym) {
    group_scale_zero(-ma, ma, a.qp, a.sym, scale, zero);
  } else {
    group_scale_zero(mn, mx, a.qp, a.sym, scale, zero);
  }
  if (valid && a.scales) {
    a.scales[row * a.n_groups + gi] = scale;
    a.zeros[row * a.n_groups + gi] = zero;
  }
}

// One 128-column block of the sweep for R groups of 32 rows: lane l of every
// warp of row group g works on row 32 (R blockIdx.x + g) + l.  Columns are
// taken in sub-blocks of 32.  Per group, the warp of role 0 runs the serial
// part: the sub-block's columns one by one in registers, each column's scaled
// error applied at once to the later columns of the sub-block (U tile
// broadcast from shared memory).  The sub-block's 32 errors must then reach
// the block's remaining columns, which live in the group's shared-memory row
// buffer (one column of 32 rows per ws row):
//   critical: the group's four warps update the next sub-block's columns (the
//             whole next group when a 64-column group starts there), then
//             role 0 goes on;
//   look-ahead: while role 0 works on that sub-block, roles 1-3 update the
//             columns beyond it and store the previous sub-block's
//             dequantized values, errors and codes; the look-ahead warps of
//             all groups together stage the U tiles the chains and the next
//             critical step read.
// Every column still receives the updates of all earlier columns in
// increasing order, one fmaf each, so the result does not depend on the
// split.  G: group size when it divides 128 (4..128), 0 when groups span
// blocks.
constexpr int SR_THREADS = 128;
constexpr int SR_CP = 2 * SW_SUB + 4;  // pitch of the critical U tile (up to 64 columns)

// The block's band U[b0:b1, b0:b1], staged in dynamic shared memory:
// us[j * SW_BLOCK + i] = U[b0 + i][b0 + j] for i <= j (the zero triangle is
// not copied and never read).
constexpr size_t SR_BAND_BYTES = (size_t)SW_BLOCK * SW_BLOCK * 4;  // 64 KB
// Per row group of 32 rows: the row buffer ws, two sub-blocks of errors es and
// of packed codes cs (16-byte multiples, so every group's buffers stay aligned).
constexpr size_t SR_WS_BYTES = (size_t)SW_BLOCK * SW_WP * 4;        // 16,896
constexpr size_t SR_ES_BYTES = (size_t)2 * SW_SUB * SW_WP * 4;      // 8,448
constexpr size_t SR_CS_BYTES = (size_t)2 * (SW_SUB / 4) * 32 * 4;  // 2,048
constexpr size_t SR_GROUP_BYTES = SR_WS_BYTES + SR_ES_BYTES + SR_CS_BYTES;
static_assert(SR_WS_BYTES % 16 == 0 && SR_ES_BYTES % 16 == 0 && SR_CS_BYTES % 16 == 0,
              "row-group buffers must keep 16-byte alignment");
// dynamic shared memory of a block step with R row groups per CTA
constexpr size_t sr_smem_bytes(int r) { return SR_BAND_BYTES + (size_t)r * SR_GROUP_BYTES; }

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gmem_src)
               : "memory");
}

template <int G, int R>
__global__ void __launch_bounds__(SR_THREADS * R) sweep_rows_kernel(SweepArgs a) {
  constexpr int GD = (G > 0) ? G : 1;  // divisor-safe group size for the G = 0 instance
  // dynamic: the band (SR_BAND_BYTES), then each row group's buffers (SR_GROUP_BYTES)
  extern __shared__ __align__(16) float us[];
  __shared__ __align__(16) float tile[2][SW_SUB * SW_TP];  // U inside sub-block s, [k][t]
  __shared__ __align__(16) float ucrit[SW_SUB * SR_CP];    // U rows of sub-block s, critical columns
  __shared__ float rinv[SW_BLOCK];
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // row group grp = warps 4 grp .. 4 grp + 3; its column-chain warp (role 0)
  // is warp 4 grp + grp % 4, so the R chains sit on different schedulers
  const int grp = wid >> 2;
  const int warp = (wid - grp) & 3;
  char* gbase = reinterpret_cast<char*>(us) + SR_BAND_BYTES + (size_t)grp * SR_GROUP_BYTES;
  float* ws = reinterpret_cast<float*>(gbase);            // ws[j][lane]: column j of the rows
  float (*es)[SW_SUB * SW_WP] =                           // errors of sub-block s, [k][lane]
      reinterpret_cast<float (*)[SW_SUB * SW_WP]>(gbase + SR_WS_BYTES);
  uint32_t (*cs)[(SW_SUB / 4) * 32] =                     // packed codes of sub-block s
      reinterpret_cast<uint32_t (*)[(SW_SUB / 4) * 32]>(gbase + SR_WS_BYTES + SR_ES_BYTES);
  const int bw = a.bw;
  const int64_t row = ((int64_t)blockIdx.x * R + grp) * 32 + lane;
  const bool valid = row < a.m;
  float* wrow = valid ? a.wp + row * a.ldp + a.b0 : nullptr;
  const int nsub = (bw + SW_SUB - 1) / SW_SUB;

  // width of the critical update after sub-block s: the next sub-block, or
  // the whole next group when a group wider than 32 columns starts there
  auto crit_width = [&](int s) -> int {
    const int c1 = SW_SUB * (s + 1);
    if (c1 >= bw) return 0;
    const int wdt = (G > SW_SUB && G <= SW_BLOCK && c1 % GD == 0) ? G : SW_SUB;
    return min(wdt, bw - c1);
  };
  // U inside sub-block s: tile[s & 1][k][t] = U[b0 + c0 + k][b0 + c0 + t]
  auto stage_tile = [&](int s, int t0, int nt) {
    const int c0 = SW_SUB * s;
    for (int e = t0; e < SW_SUB * (SW_SUB / 4); e += nt) {
      const int t = e / (SW_SUB / 4), q = e % (SW_SUB / 4);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c0 + t < bw) v = *(reinterpret_cast<const float4*>(us + (c0 + t) * SW_BLOCK + c0) + q);
      float* dst = &tile[s & 1][(4 * q) * SW_TP + t];
      dst[0] = v.x;
      dst[SW_TP] = v.y;
      dst[2 * SW_TP] = v.z;
      dst[3 * SW_TP] = v.w;
    }
  };
  // U rows of sub-block s for its critical columns: ucrit[k][t] = U[b0 + c0 + k][b0 + c1 + t]
  auto stage_crit = [&](int s, int t0, int nt) {
    const int c0 = SW_SUB * s, c1 = c0 + SW_SUB, wdt = crit_width(s);
    for (int e = t0; e < wdt * (SW_SUB / 4); e += nt) {
      const int t = e / (SW_SUB / 4), q = e % (SW_SUB / 4);
      const float4 v = *(reinterpret_cast<const float4*>(us + (c1 + t) * SW_BLOCK + c0) + q);
      float* dst = &ucrit[(4 * q) * SR_CP + t];
      dst[0] = v.x;
      dst[SR_CP] = v.y;
      dst[2 * SR_CP] = v.z;
      dst[3 * SR_CP] = v.w;
    }
  };
  // column j -= sum_k ev[k] U[b0 + c0 + k][b0 + j], k increasing (U broadcast from the band)
  // columns j0, j0 + dj, ... (nj <= 4 of them) -= sum_k ev[k] U[b0 + c0 + k][b0 + j],
  // k increasing, U broadcast from the band: independent chains side by side
  // (each column still adds its 32 terms in increasing k), so the FMA latency
  // of one chain hides behind the others
  auto update_cols_from_band = [&](const float (&ev)[SW_SUB], int c0, int j0, int dj, int nj) {
    constexpr int NJ = 4;
    float v[NJ];
    const float4* u4[NJ];
#pragma unroll
    for (int c = 0; c < NJ; ++c) {
      const int j = (c < nj) ? j0 + c * dj : j0;
      u4[c] = reinterpret_cast<const float4*>(us + j * SW_BLOCK + c0);
      v[c] = ws[j * SW_WP + lane];
    }
#pragma unroll
    for (int kc = 0; kc < SW_SUB / 4; ++kc) {
#pragma unroll
      for (int c = 0; c < NJ; ++c) {
        const float4 u = u4[c][kc];
        v[c] = fmaf(-ev[4 * kc + 0], u.x, v[c]);
        v[c] = fmaf(-ev[4 * kc + 1], u.y, v[c]);
        v[c] = fmaf(-ev[4 * kc + 2], u.z, v[c]);
        v[c] = fmaf(-ev[4 * kc + 3], u.w, v[c]);
      }
    }
#pragma unroll
    for (int c = 0; c < NJ; ++c)
      if (c < nj) ws[(j0 + c * dj) * SW_WP + lane] = v[c];
  };
  // sub-block s's results to global memory (dequantized values, errors, codes)
  auto store_sub = [&](int s, int t0, int nt) {
    if (!valid) return;
    const int c0 = SW_SUB * s;
    float* erow = a.err + row * a.ld_err + c0;
    uint8_t* crow = a.cp + row * a.ldp + a.b0 + c0;
    const bool full = c0 + SW_SUB <= bw;
    for (int q = t0; q < SW_SUB / 4; q += nt) {
      if (full) {
        *reinterpret_cast<float4*>(wrow + c0 + 4 * q) =
            make_float4(ws[(c0 + 4 * q) * SW_WP + lane], ws[(c0 + 4 * q + 1) * SW_WP + lane],
                        ws[(c0 + 4 * q + 2) * SW_WP + lane], ws[(c0 + 4 * q + 3) * SW_WP + lane]);
        const float* e = es[s & 1];
        *reinterpret_cast<float4*>(erow + 4 * q) =
            make_float4(e[(4 * q) * SW_WP + lane], e[(4 * q + 1) * SW_WP + lane],
                        e[(4 * q + 2) * SW_WP + lane], e[(4 * q + 3) * SW_WP + lane]);
        *reinterpret_cast<uint32_t*>(crow + 4 * q) = cs[s & 1][q * 32 + lane];
      } else {
        for (int t = 0; t < 4; ++t) {
          const int k = 4 * q + t;
          if (c0 + k < bw) {
            wrow[c0 + k] = ws[(c0 + k) * SW_WP + lane];
            erow[k] = es[s & 1][k * SW_WP + lane];
            crow[k] = (uint8_t)(cs[s & 1][q * 32 + lane] >> (8 * t));
          }
        }
      }
    }
  };

  // ---- prologue (all warps): the band (asynchronously), the row block,
  // reciprocal pivots, the first tiles
  constexpr int NT = SR_THREADS * R;
  for (int c = threadIdx.x; c < bw * (SW_BLOCK / 4); c += NT) {
    const int j = c / (SW_BLOCK / 4), q = c % (SW_BLOCK / 4);
    if (4 * q <= j) cp_async16(us + j * SW_BLOCK + 4 * q, a.ubt + (int64_t)j * a.ldub + 4 * q);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  if (valid) {
    // warp w loads columns [32 w, 32 w + 32): eight float4 loads in flight per lane
    float4 v[SW_SUB / 4];
#pragma unroll
    for (int q = 0; q < SW_SUB / 4; ++q) {
      const int j = SW_SUB * warp + 4 * q;
      v[q] = (j < bw) ? *reinterpret_cast<const float4*>(wrow + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int q = 0; q < SW_SUB / 4; ++q) {
      const int j = SW_SUB * warp + 4 * q;
      ws[(j + 0) * SW_WP + lane] = v[q].x;
      ws[(j + 1) * SW_WP + lane] = v[q].y;
      ws[(j + 2) * SW_WP + lane] = v[q].z;
      ws[(j + 3) * SW_WP + lane] = v[q].w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < SW_SUB; ++k) ws[(SW_SUB * warp + k) * SW_WP + lane] = 0.f;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  for (int i = threadIdx.x; i < SW_BLOCK; i += NT)
    rinv[i] = (i < bw) ? 1.f / us[i * SW_BLOCK + i] : 0.f;
  stage_tile(0, threadIdx.x, NT);
  float scale = 1.f, zero = 0.f;  // warp 0: the current group's parameters
  if (G == 0 && valid) {
    scale = a.big_scale[row];
    zero = a.big_zero[row];
  }
  __syncthreads();

  for (int s = 0; s < nsub; ++s) {
    const int c0 = SW_SUB * s;
    const int w_prev = (s > 0) ? crit_width(s - 1) : 0;
    if (warp == 0) {
      // ---- the sub-block's columns, in registers
      const float* tl = tile[s & 1];
      float w[SW_SUB], e[SW_SUB];
      uint32_t cw[SW_SUB / 4];
#pragma unroll
      for (int k = 0; k < SW_SUB; ++k) w[k] = (c0 + k < bw) ? ws[(c0 + k) * SW_WP + lane] : 0.f;
#pragma unroll
      for (int q = 0; q < SW_SUB / 4; ++q) cw[q] = 0u;
#pragma unroll
      for (int k = 0; k < SW_SUB; ++k) {
        const int i = c0 + k;
        if (i >= bw) {
          e[k] = 0.f;
          continue;
        }
        // group parameters at the group's first column, from the current values
        if (G > 0 && G <= SW_SUB && (k % GD) == 0) {
          float mn = INFINITY, mx = -INFINITY, ma = 0.f;
#pragma unroll
          for (int t = k; t < k + GD && t < SW_SUB; ++t) {
            mn = fminf(mn, w[t]);
            mx = fmaxf(mx, w[t]);
            ma = fmaxf(ma, fabsf(w[t]));
          }
          sweep_group_params(a, row, valid, (a.b0 + i) / GD, mn, mx, ma, scale, zero);
        }
        if (G > SW_SUB && k == 0 && (c0 % GD) == 0) {
          float mn = INFINITY, mx = -INFINITY, ma = 0.f;
#pragma unroll
          for (int t = 0; t < SW_SUB; ++t) {
            mn = fminf(mn, w[t]);
            mx = fmaxf(mx, w[t]);
            ma = fmaxf(ma, fabsf(w[t]));
          }
          for (int j = c0 + SW_SUB; j < c0 + G; ++j) {
            const float v = ws[j * SW_WP + lane];
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
            ma = fmaxf(ma, fabsf(v));
          }
          sweep_group_params(a, row, valid, (a.b0 + i) / GD, mn, mx, ma, scale, zero);
        }
        float dq;
        const float q = quantize_one(w[k], scale, zero, a.qp, dq);
        const bool prop = a.b0 + i >= a.noprop_cols;
        e[k] = prop ? __fmul_rn(__fsub_rn(w[k], dq), rinv[i]) : 0.f;
        w[k] = dq;
        cw[k >> 2] |= ((uint32_t)(int)(q - a.qp.qmin) & 0xffu) << (8 * (k & 3));
#pragma unroll
        for (int q4 = 0; q4 < SW_SUB / 4; ++q4) {
          if (4 * q4 + 3 > k) {
            const float4 u4 = *reinterpret_cast<const float4*>(&tl[k * SW_TP + 4 * q4]);
            const float uu[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
            for (int t = 0; t < 4; ++t)
              if (4 * q4 + t > k) w[4 * q4 + t] = fmaf(-e[k], uu[t], w[4 * q4 + t]);
          }
        }
      }
      // publish: dequantized values into the row buffer, errors and codes
#pragma unroll
      for (int k = 0; k < SW_SUB; ++k) {
        if (c0 + k < bw) ws[(c0 + k) * SW_WP + lane] = w[k];
        es[s & 1][k * SW_WP + lane] = e[k];
      }
#pragma unroll
      for (int q = 0; q < SW_SUB / 4; ++q) cs[s & 1][q * 32 + lane] = cw[q];
    } else {
      // ---- look-ahead (roles 1-3 of every row group; the U tiles are
      // staged by the look-ahead warps of all groups together)
      const int lw = warp - 1, lt = (grp * 3 + lw) * 32 + lane;
      if (s > 0) {
        // sub-block s-1's errors reach the columns past its critical update
        float ev[SW_SUB];
#pragma unroll
        for (int k = 0; k < SW_SUB; ++k) ev[k] = es[(s - 1) & 1][k * SW_WP + lane];
        constexpr int LW = SR_THREADS / 32 - 1;  // look-ahead warps
        for (int j = SW_SUB * s + w_prev + lw; j < bw; j += 4 * LW)
          update_cols_from_band(ev, SW_SUB * (s - 1), j, LW, min(4, (bw - j + LW - 1) / LW));
        store_sub(s - 1, lw, SR_THREADS / 32 - 1);
      }
      if (s + 1 < nsub) stage_tile(s + 1, lt, (SR_THREADS - 32) * R);
      stage_crit(s, lt, (SR_THREADS - 32) * R);
    }
    __syncthreads();
    // ---- critical: sub-block s's errors reach the next critical columns (all warps)
    const int wc = crit_width(s);
    if (wc > 0) {
      float ev[SW_SUB];
#pragma unroll
      for (int k = 0; k < SW_SUB; ++k) ev[k] = es[s & 1][k * SW_WP + lane];
      constexpr int NW = SR_THREADS / 32;
      // columns t, t + NW, t + 2 NW, t + 3 NW together: four independent chains
      for (int t = warp; t < wc; t += 4 * NW) {
        float v[4];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          v[c] = (t + c * NW < wc) ? ws[(c0 + SW_SUB + t + c * NW) * SW_WP + lane] : 0.f;
#pragma unroll
        for (int k = 0; k < SW_SUB; ++k) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            v[c] = fmaf(-ev[k], ucrit[k * SR_CP + min(t + c * NW, wc - 1)], v[c]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (t + c * NW < wc) ws[(c0 + SW_SUB + t + c * NW) * SW_WP + lane] = v[c];
      }
    }
    __syncthreads();
  }
  // the last sub-block's results (its look-ahead step never came)
  store_sub(nsub - 1, warp, SR_THREADS / 32);
}

// Single-warp form of the block step, for grids too large to keep four-warp
// CTAs resident in one wave: lane l owns row 32 * blockIdx.x + l.
// Columns are taken in sub-blocks of 32 held in registers; inside a sub-block
// each column's scaled error is applied at once to the later columns
// (right-looking, U tile broadcast from shared memory), and after the
// sub-block its 32 errors are applied to the block's remaining columns, which
// live in a lane-private shared-memory row buffer.  Every column therefore
// receives the updates of all earlier columns in increasing order, one fmaf
// each.  G: group size when it divides 128 (4..128), 0 when groups span blocks.
template <int G>
__global__ void __launch_bounds__(32) sweep_rows1_kernel(SweepArgs a) {
  constexpr int GD = (G > 0) ? G : 1;  // divisor-safe group size for the G = 0 instance
  __shared__ float ws[SW_BLOCK * SW_WP];
  __shared__ __align__(16) float tile[SW_SUB * SW_TP];
  __shared__ float rinv[SW_BLOCK];
  // U rows the current sub-block's errors update: stg[j - c0 - 32][k] = U[b0 + c0 + k][b0 + j]
  __shared__ __align__(16) float stg[(SW_BLOCK - SW_SUB) * SW_SUB];
  const int lane = threadIdx.x;
  const int bw = a.bw;
  const float* __restrict__ ubt = a.ubt;
  for (int i = lane; i < SW_BLOCK; i += 32)
    rinv[i] = (i < bw) ? 1.f / ubt[(int64_t)i * a.ldub + i] : 0.f;
  const int64_t row = (int64_t)blockIdx.x * 32 + lane;
  const bool valid = row < a.m;
  float* wrow = valid ? a.wp + row * a.ldp + a.b0 : nullptr;
  if (valid) {
    // the row's block in two batches of 16 loads in flight (not one load per round trip)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float4 v[SW_BLOCK / 8];
#pragma unroll
      for (int q = 0; q < SW_BLOCK / 8; ++q) {
        const int j = half * (SW_BLOCK / 2) + 4 * q;
        v[q] = (j < bw) ? *reinterpret_cast<const float4*>(wrow + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int q = 0; q < SW_BLOCK / 8; ++q) {
        const int j = half * (SW_BLOCK / 2) + 4 * q;
        ws[(j + 0) * SW_WP + lane] = v[q].x;
        ws[(j + 1) * SW_WP + lane] = v[q].y;
        ws[(j + 2) * SW_WP + lane] = v[q].z;
        ws[(j + 3) * SW_WP + lane] = v[q].w;
      }
    }
  }
  float scale = 1.f, zero = 0.f;
  if (G == 0 && valid) {
    scale = a.big_scale[row];
    zero = a.big_zero[row];
  }
  __syncwarp();

  for (int c0 = 0; c0 < bw; c0 += SW_SUB) {
    // start copying the U rows for this sub-block's trailing update; they land
    // while the column loop below runs
    const int trail = bw - c0 - SW_SUB;
    for (int ch = lane; ch < trail * (SW_SUB / 4); ch += 32) {
      const int r = ch / (SW_SUB / 4), part = ch % (SW_SUB / 4);
      const float* src = ubt + (int64_t)(c0 + SW_SUB + r) * a.ldub + c0 + 4 * part;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                       (uint32_t)__cvta_generic_to_shared(stg + r * SW_SUB + 4 * part)),
                   "l"(src)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    // tile[k][t] = U[b0 + c0 + k][b0 + c0 + t]  (lane t copies its row of the band)
    if (c0 + lane < bw) {
      const float4* src = reinterpret_cast<const float4*>(ubt + (int64_t)(c0 + lane) * a.ldub + c0);
#pragma unroll
      for (int q = 0; q < SW_SUB / 4; ++q) {
        const float4 v = __ldg(src + q);
        tile[(4 * q + 0) * SW_TP + lane] = v.x;
        tile[(4 * q + 1) * SW_TP + lane] = v.y;
        tile[(4 * q + 2) * SW_TP + lane] = v.z;
        tile[(4 * q + 3) * SW_TP + lane] = v.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < SW_SUB; ++k) tile[k * SW_TP + lane] = 0.f;
    }
    __syncwarp();
    float w[SW_SUB], e[SW_SUB];
    uint32_t cw[SW_SUB / 4];
#pragma unroll
    for (int k = 0; k < SW_SUB; ++k) w[k] = (c0 + k < bw) ? ws[(c0 + k) * SW_WP + lane] : 0.f;
#pragma unroll
    for (int q = 0; q < SW_SUB / 4; ++q) cw[q] = 0u;

#pragma unroll
    for (int k = 0; k < SW_SUB; ++k) {
      const int i = c0 + k;
      if (i >= bw) {
        e[k] = 0.f;
        continue;
      }
      // group parameters at the group's first column, from the current values
      if (G > 0 && G <= SW_SUB && (k % GD) == 0) {
        float mn = INFINITY, mx = -INFINITY, ma = 0.f;
#pragma unroll
        for (int t = k; t < k + GD && t < SW_SUB; ++t) {
          mn = fminf(mn, w[t]);
          mx = fmaxf(mx, w[t]);
          ma = fmaxf(ma, fabsf(w[t]));
        }
        sweep_group_params(a, row, valid, (a.b0 + i) / GD, mn, mx, ma, scale, zero);
      }
      if (G > SW_SUB && k == 0 && (c0 % GD) == 0) {
        float mn = INFINITY, mx = -INFINITY, ma = 0.f;
#pragma unroll
        for (int t = 0; t < SW_SUB; ++t) {
          mn = fminf(mn, w[t]);
          mx = fmaxf(mx, w[t]);
          ma = fmaxf(ma, fabsf(w[t]));
        }
        for (int j = c0 + SW_SUB; j < c0 + G; ++j) {
          const float v = ws[j * SW_WP + lane];
          mn = fminf(mn, v);
          mx = fmaxf(mx, v);
          ma = fmaxf(ma, fabsf(v));
        }
        sweep_group_params(a, row, valid, (a.b0 + i) / GD, mn, mx, ma, scale, zero);
      }
      float dq;
      const float q = quantize_one(w[k], scale, zero, a.qp, dq);
      const bool prop = a.b0 + i >= a.noprop_cols;
      e[k] = prop ? __fmul_rn(__fsub_rn(w[k], dq), rinv[i]) : 0.f;
      w[k] = dq;
      cw[k >> 2] |= ((uint32_t)(int)(q - a.qp.qmin) & 0xffu) << (8 * (k & 3));
#pragma unroll
      for (int q4 = 0; q4 < SW_SUB / 4; ++q4) {
        if (4 * q4 + 3 > k) {
          const float4 u4 = *reinterpret_cast<const float4*>(&tile[k * SW_TP + 4 * q4]);
          const float uu[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
          for (int t = 0; t < 4; ++t)
            if (4 * q4 + t > k) w[4 * q4 + t] = fmaf(-e[k], uu[t], w[4 * q4 + t]);
        }
      }
    }

    if (valid) {
      float* erow = a.err + row * a.ld_err + c0;
      uint8_t* crow = a.cp + row * a.ldp + a.b0 + c0;
      if (c0 + SW_SUB <= bw) {
#pragma unroll
        for (int q = 0; q < SW_SUB / 4; ++q) {
          *reinterpret_cast<float4*>(wrow + c0 + 4 * q) =
              make_float4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
          *reinterpret_cast<float4*>(erow + 4 * q) =
              make_float4(e[4 * q], e[4 * q + 1], e[4 * q + 2], e[4 * q + 3]);
          *reinterpret_cast<uint32_t*>(crow + 4 * q) = cw[q];
        }
      } else {
#pragma unroll
        for (int k = 0; k < SW_SUB; ++k) {
          if (c0 + k < bw) {
            wrow[c0 + k] = w[k];
            erow[k] = e[k];
            crow[k] = (uint8_t)(cw[k >> 2] >> (8 * (k & 3)));
          }
        }
      }
    }

    // the block's later columns: ws[j] -= sum_k e[k] U[c0 + k][j], k increasing
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    const float4* ub4 = reinterpret_cast<const float4*>(stg);
    for (int j0 = c0 + SW_SUB; j0 < bw; j0 += 4) {
      float v[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) v[jj] = ws[(j0 + jj) * SW_WP + lane];
#pragma unroll
      for (int kc = 0; kc < SW_SUB / 4; ++kc) {
        float4 u4[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          u4[jj] = (j0 + jj < bw) ? ub4[(j0 + jj - c0 - SW_SUB) * (SW_SUB / 4) + kc]
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          v[jj] = fmaf(-e[4 * kc + 0], u4[jj].x, v[jj]);
          v[jj] = fmaf(-e[4 * kc + 1], u4[jj].y, v[jj]);
          v[jj] = fmaf(-e[4 * kc + 2], u4[jj].z, v[jj]);
          v[jj] = fmaf(-e[4 * kc + 3], u4[jj].w, v[jj]);
        }
      }
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) ws[(j0 + jj) * SW_WP + lane] = v[jj];
    }
    __syncwarp();
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

// Super-block width for a group size (see the file comment).
inline int sweep_super(int group_size) {
  const bool fits = group_size <= SW_BLOCK || SW_SUPER % group_size == 0 ||
                    group_size % SW_SUPER == 0;
  return fits ? SW_SUPER : SW_BLOCK;
}

// Byte offset of the transposed U band (after wp, cp, err, bscale, bzero).
inline int64_t sweep_ubt_offset(int64_t m, int64_t n) {
  int64_t ldp = round4(n);
  int64_t off = m * ldp * 4 + ((m * ldp + 15) & ~int64_t(15)) + m * SW_SUPER * 4 + 2 * m * 4;
  return (off + 255) & ~int64_t(255);
}

// ubt holds a band [<= 512, 128] or the far block U[s0:s1, s1:]^T [n - s1, 512].
// Only meaningful for shapes that pass sweep_shape_ok (no int64 overflow).
int64_t sweep_ws_bytes(int64_t m, int64_t n) {
  return sweep_ubt_offset(m, n) + n * SW_SUPER * 4 + 256;
}

// Largest n whose row (float value + code per column) fits the shared-memory
// row buffer of the gather / scatter kernels.
constexpr int64_t kSweepMaxCols = (220 * 1024 - 64) / 5;

// Rejects shapes whose workspace size would not fit in int64: the workspace
// is below m * (5 * round4(n) + 4 * 512 + 8) + n * 2048 + 768 bytes.
int sweep_shape_ok(const char* who, int64_t m, int64_t n) {
  GQ_REQUIRE(m >= 0 && n >= 0, "%s: negative shape %lld x %lld", who, (long long)m, (long long)n);
  GQ_REQUIRE(n <= kSweepMaxCols, "%s: n=%lld exceeds the row buffer (at most %lld columns)", who,
             (long long)n, (long long)kSweepMaxCols);
  const int64_t per_row = 8 * round4(n) + 8 * SW_SUPER + 64;
  GQ_REQUIRE(m <= (INT64_MAX / 2) / per_row, "%s: m=%lld rows is too large", who, (long long)m);
  return GQ_OK;
}

int transpose2d(const float* src, int64_t rows, int64_t cols, int64_t lds, float* dst, int64_t ldd,
                cudaStream_t st);

// Row groups per CTA of the four-warp block step (gq_set_sweep_row_groups):
// 0 picks by row count, 1, 2 or 4 force that many, -1 forces the one-warp
// kernel.
static std::atomic<int> g_row_groups{0};

// The four-warp block step takes the band and its row groups' buffers in
// dynamic shared memory above the default 48 KB; allowed once per (device,
// instance).
template <int G, int R>
static int launch_rows4(const SweepArgs& a, unsigned grid, cudaStream_t st) {
  // setting the attribute twice (two threads racing here) is harmless
  static std::atomic<int> done_dev{-1};
  int dev = 0;
  GQ_CHECK_CUDA(cudaGetDevice(&dev));
  if (done_dev.load(std::memory_order_relaxed) != dev) {
    GQ_CHECK_CUDA(cudaFuncSetAttribute(sweep_rows_kernel<G, R>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)sr_smem_bytes(R)));
    done_dev.store(dev, std::memory_order_relaxed);
  }
  sweep_rows_kernel<G, R><<<grid, SR_THREADS * R, sr_smem_bytes(R), st>>>(a);
  return GQ_OK;
}

template <int R>
static int launch_rows4_g(int group_size, const SweepArgs& a, unsigned grid, cudaStream_t st) {
  switch (group_size) {
    case 4: return launch_rows4<4, R>(a, grid, st);
    case 8: return launch_rows4<8, R>(a, grid, st);
    case 16: return launch_rows4<16, R>(a, grid, st);
    case 32: return launch_rows4<32, R>(a, grid, st);
    case 64: return launch_rows4<64, R>(a, grid, st);
    case 128: return launch_rows4<128, R>(a, grid, st);
    default: return launch_rows4<0, R>(a, grid, st);
  }
}

static int launch_rows1_g(int group_size, const SweepArgs& a, unsigned grid, cudaStream_t st) {
  switch (group_size) {
    case 4: sweep_rows1_kernel<4><<<grid, 32, 0, st>>>(a); break;
    case 8: sweep_rows1_kernel<8><<<grid, 32, 0, st>>>(a); break;
    case 16: sweep_rows1_kernel<16><<<grid, 32, 0, st>>>(a); break;
    case 32: sweep_rows1_kernel<32><<<grid, 32, 0, st>>>(a); break;
    case 64: sweep_rows1_kernel<64><<<grid, 32, 0, st>>>(a); break;
    case 128: sweep_rows1_kernel<128><<<grid, 32, 0, st>>>(a); break;
    default: sweep_rows1_kernel<0><<<grid, 32, 0, st>>>(a); break;
  }
  return GQ_OK;
}

// Row groups per CTA for m rows on `sms` SMs; 0 selects the one-warp kernel.
// One group per CTA (110 KB of shared memory, two CTAs per SM) while those
// fit in one wave; four (194 KB, one per SM) while those do; beyond that the
// one-warp kernel, whose 34 KB CTAs keep a wave of them resident.
static int pick_row_groups(int64_t m, int sms) {
  const int forced = g_row_groups.load(std::memory_order_relaxed);
  if (forced != 0) return forced < 0 ? 0 : forced;
  const int64_t rows32 = ceil_div(m, 32);
  if (rows32 <= 2 * (int64_t)sms) return 1;
  if (rows32 <= 4 * (int64_t)sms) return 4;
  return 0;
}

}  // namespace gq

extern "C" {

int64_t gq_gptq_sweep_workspace_size(int64_t m, int64_t n) { return gq::sweep_ws_bytes(m, n); }

int gq_set_sweep_row_groups(int r) {
  GQ_REQUIRE(r == -1 || r == 0 || r == 1 || r == 2 || r == 4,
             "gq_set_sweep_row_groups: %d is not one of -1, 0, 1, 2, 4", r);
  gq::g_row_groups.store(r, std::memory_order_relaxed);
  return GQ_OK;
}

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
  GQ_REQUIRE((w != nullptr || m == 0) && ldw >= n, "gq_gptq_sweep: bad w");
  GQ_REQUIRE((group0_scale == nullptr) == (group0_zero == nullptr),
             "gq_gptq_sweep: group0_scale and group0_zero must both be given or both NULL");
  GQ_REQUIRE((scales == nullptr) == (zeros == nullptr),
             "gq_gptq_sweep: scales and zeros must both be given or both NULL");
  GQ_TRY(sweep_shape_ok("gq_gptq_sweep", m, n));
  GQ_REQUIRE(workspace_bytes >= sweep_ws_bytes(m, n), "gq_gptq_sweep: workspace too small");
  GQ_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
             "gq_gptq_sweep: workspace must be 256-byte aligned");
  if (n == 0) return GQ_OK;
  cudaStream_t st = as_stream(stream);
  if (m == 0) {
    // no rows (e.g. an empty row shard): the group index of every column is
    // still an output, and it depends only on the permutation
    if (g_idx) {
      g_idx_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(perm, n, group_size, g_idx);
      GQ_TRY(check_launch("g_idx"));
    }
    return GQ_OK;
  }
  const int64_t ldp = round4(n);
  char* ws = reinterpret_cast<char*>(workspace);
  float* wp = reinterpret_cast<float*>(ws);
  uint8_t* cp = reinterpret_cast<uint8_t*>(ws + m * ldp * 4);
  float* err = reinterpret_cast<float*>(ws + m * ldp * 4 + ((m * ldp + 15) & ~int64_t(15)));
  float* bscale = err + m * SW_SUPER;
  float* bzero = bscale + m;
  float* ubt = reinterpret_cast<float*>(ws + sweep_ubt_offset(m, n));  // [n, 512]
  const int super_w = sweep_super(group_size);

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
  a.wp = wp; a.cp = cp; a.ubt = ubt; a.ldub = super_w;
  a.ld_err = super_w;
  a.m = m; a.n = n; a.ldp = ldp;
  a.n_groups = (int)(n / group_size);
  a.qp = make_qparams(w_bits, sym); a.sym = sym;
  a.noprop_cols = noprop_cols;
  a.group0_scale = group0_scale; a.group0_zero = group0_zero;
  a.big_scale = bscale; a.big_zero = bzero;
  a.scales = scales; a.zeros = zeros;
  int dev = 0, sms = 0;
  GQ_CHECK_CUDA(cudaGetDevice(&dev));
  GQ_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int row_groups = pick_row_groups(m, sms);
  const unsigned grid = (unsigned)ceil_div(m, 32 * (int64_t)std::max(1, row_groups));
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
    const int64_t s0 = b0 - b0 % super_w;
    const int64_t s1 = std::min<int64_t>(n, s0 + super_w);
    a.b0 = b0;
    a.bw = bw;
    a.err = err + (b0 - s0);
    if (b0 == s0) {
      // U[s0:s1, s0:n] transposed: the block steps read U's super-block rows
      // as contiguous runs, and both GEMMs get their U operand K-major
      // (tensor-core path)
      GQ_TRY(transpose2d(u + s0 * ldu + s0, s1 - s0, n - s0, ldu, ubt, super_w, st));
    }
    a.ubt = ubt + (b0 - s0) * super_w + (b0 - s0);
    switch (row_groups) {
      case 1: GQ_TRY(launch_rows4_g<1>(group_size, a, grid, st)); break;
      case 2: GQ_TRY(launch_rows4_g<2>(group_size, a, grid, st)); break;
      case 4: GQ_TRY(launch_rows4_g<4>(group_size, a, grid, st)); break;
      default: GQ_TRY(launch_rows1_g(group_size, a, grid, st)); break;
    }
    GQ_TRY(check_launch("sweep_rows"));
    const int64_t b1 = b0 + bw;
    if (b1 < s1) {
      // near: wp[:, b1:s1] -= err_block @ U[b0:b1, b1:s1]
      GQ_TRY(sgemm(0, 1, m, s1 - b1, bw, -1.f, a.err, super_w, a.ubt + (int64_t)bw * super_w,
                   super_w, 1.f, wp + b1, ldp, 0, st));
    }
    if (b1 == s1 && s1 < n) {
      // far: wp[:, s1:] -= err @ U[s0:s1, s1:]
      GQ_TRY(sgemm(0, 1, m, n - s1, s1 - s0, -1.f, err, super_w, ubt + (s1 - s0) * super_w,
                   super_w, 1.f, wp + s1, ldp, 0, st));
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
