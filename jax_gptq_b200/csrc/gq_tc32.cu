// Float32-accurate GEMM on the tcgen05 tensor cores:
//   C = alpha * A * B^T + beta * C,  A [M, K] and B [N, K] row-major (both
//   K-major operands, "NT").  Callers with a [K, N] B transpose it first: for
//   32-bit MN-major operands the UMMA expects the 32-byte-atom variant of the
//   128-byte swizzle, not the layout a SWIZZLE_128B TMA load writes.
//
// kind::tf32 multiplies keep 10 mantissa bits, so each operand tile is split
// in shared memory into hi = x with the low 13 mantissa bits cleared (exactly
// representable in tf32) and lo = x - hi (exact in fp32), and every k-step
// issues three MMAs, lo*hi + hi*lo + hi*hi, into the fp32 TMEM accumulator.
// The dropped lo*lo term and the tf32 rounding of lo leave a relative error
// near 2^-21 per product -- close to float32 GEMM accuracy.
//
// One CTA per SM, persistent over 128 x 128 output tiles, 3-stage ring of
// 32-float-deep (128-byte) k-slices:
//   warp 0     TMA producer (one thread)
//   warp 1     MMA issuer (one thread), 2 TMEM accumulators of 128 columns
//   warps 2-5  lo converters (lo = raw - hi to its own buffer; the raw tile is the hi operand)
//   warps 6-9  epilogue: tcgen05.ld, then for beta 0 / 1 swizzled 32 x 32
//              chunks written by TMA tensor stores / fp32 reduce-adds (no
//              read of C by the SM), for other beta per-row loads and stores
// All waits are bounded (timeout -> device status word, no hang); no
// multicast loads.
#include <cuda.h>

#include "gq_common.cuh"

namespace gq {
namespace tc32 {

// This file's device status word (device variables are per translation unit
// without relocatable device code); gq_device_status() reads it.
static __device__ int g_device_status = 0;
// this file's bound on every mbarrier wait (gq_set_wait_limit_ns)
static __device__ uint64_t g_wait_limit_ns = kWaitLimitNs;

int read_status(int reset, int* out) {
  int v = 0;
  GQ_CHECK_CUDA(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)));
  if (reset) {
    int z = 0;
    GQ_CHECK_CUDA(cudaMemcpyToSymbol(g_device_status, &z, sizeof(int)));
  }
  *out = v;
  return GQ_OK;
}

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 4;
constexpr int CHUNK_KB = 4;  // k-slices (x 32 of K) per TMEM accumulation
constexpr int A_BYTES = BM * BK * 4;   // 16 KB
constexpr int B_BYTES = BN * BK * 4;   // 16 KB
constexpr int STAGE_BYTES = A_BYTES + 2 * B_BYTES;  // raw A | raw B (= B hi) | B lo
constexpr int THREADS = 320;
// TMEM: two 128-column accumulators, then per stage the A slice as MMA
// operand, hi in 32 columns and lo in the next 32 (one row per lane)
constexpr int TMEM_COLS = 512;
constexpr int A_TMEM_COL0 = 2 * BN;
static_assert(A_TMEM_COL0 + STAGES * 2 * BK <= TMEM_COLS, "TMEM columns");
// epilogue staging: per epilogue warp two 32 x 32 fp32 chunks (4 KB each,
// 128-byte swizzled rows, the layout a SWIZZLE_128B tensor store reads)
constexpr int C_CHUNK_BYTES = 32 * 32 * 4;
constexpr int C_STAGE_BYTES = 4 * 2 * C_CHUNK_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + C_STAGE_BYTES + 1024 + 256;

struct Params {
  float* c;
  int64_t ldc;
  int64_t M, N, K;
  float alpha, beta;
  int uplo;
  int tri;  // 0 none, 1 A upper (k >= row0), 2 A lower (k < row0 + BM), 3 B lower (k < col0 + BN),
            // 4 B upper (k >= col0)
  int num_tiles;
  int mb, nb;
  int b_kmajor;
  int c_mode;  // 0: stores from registers (any beta); 1: TMA store (beta 0); 2: TMA add (beta 1)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > g_wait_limit_ns) {
      *abort_flag = 1;
      atomicExch(&g_device_status, GQ_DEVERR_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}
// kind::tf32: D f32 (bits 4-5 = 1), A/B tf32 (format 2), A K-major, B K- or MN-major.
__host__ __device__ constexpr uint32_t idesc(bool b_mn_major) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t id, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(id), "r"(accum));
}
// A operand from TMEM (a_tmem: column of its first k), B from shared memory.
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                             uint32_t id, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(id), "r"(accum));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// lo = x - hi with hi = x with the low 13 mantissa bits cleared (exact).  The
// MMA reads the raw fp32 tile as the hi operand: kind::tf32 ignores those 13
// bits, so the raw value and hi multiply identically.
__device__ __forceinline__ uint4 lo_part(uint4 x) {
  return make_uint4(__float_as_uint(__uint_as_float(x.x) - __uint_as_float(x.x & 0xFFFFE000u)),
                    __float_as_uint(__uint_as_float(x.y) - __uint_as_float(x.y & 0xFFFFE000u)),
                    __float_as_uint(__uint_as_float(x.z) - __uint_as_float(x.z & 0xFFFFE000u)),
                    __float_as_uint(__uint_as_float(x.w) - __uint_as_float(x.w & 0xFFFFE000u)));
}

__device__ __forceinline__ bool tile_skipped(const Params& p, int bm, int bn) {
  const int64_t row0 = (int64_t)bm * BM, col0 = (int64_t)bn * BN;
  if (p.uplo == 1 && col0 > row0 + BM - 1) return true;
  if (p.uplo == 2 && col0 + BN - 1 < row0) return true;
  return false;
}

// k-slices [kb0, kb1) of tile (bm, bn): a triangular operand whose zero
// triangle starts on a 128 boundary contributes nothing outside this range.
__device__ __forceinline__ void k_range(const Params& p, int bm, int bn, int nkb, int& kb0,
                                        int& kb1) {
  kb0 = 0;
  kb1 = nkb;
  if (p.tri == 1) kb0 = min(nkb, bm * (BM / BK));
  else if (p.tri == 2) kb1 = min(nkb, (bm + 1) * (BM / BK));
  else if (p.tri == 3) kb1 = min(nkb, (bn + 1) * (BN / BK));
  else if (p.tri == 4) kb0 = min(nkb, bn * (BN / BK));
}

__global__ void __launch_bounds__(THREADS, 1)
tf32x3_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
              const __grid_constant__ CUtensorMap map_c, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  // per stage: A raw | B raw (= B hi) | B lo
  auto a_raw = [&](int s) { return smem + s * STAGE_BYTES; };
  auto b_hi = [&](int s) { return smem + s * STAGE_BYTES + A_BYTES; };
  auto b_lo = [&](int s) { return smem + s * STAGE_BYTES + A_BYTES + B_BYTES; };
  uint8_t* c_stage = smem + STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(c_stage + C_STAGE_BYTES);
  uint64_t* conv = full + STAGES;
  uint64_t* empty = conv + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 128);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nkb = (int)((p.K + BK - 1) / BK);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x) {
        const int bm = t % p.mb, bn = t / p.mb;
        if (tile_skipped(p, bm, bn)) continue;
        int kb0, kb1;
        k_range(p, bm, bn, nkb, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
          mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
          const int k0 = kb * BK;
          tma_load_2d(&map_a, &full[stage], a_raw(stage), k0, bm * BM);
          if (p.b_kmajor) {
            tma_load_2d(&map_b, &full[stage], b_hi(stage), k0, bn * BN);
          } else {
#pragma unroll
            for (int q = 0; q < BN / 32; ++q)
              tma_load_2d(&map_b, &full[stage], b_hi(stage) + q * (BK * 128), bn * BN + q * 32, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id = idesc(!p.b_kmajor);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles && !*abort_flag; t += gridDim.x) {
        const int bm = t % p.mb, bn = t / p.mb;
        if (tile_skipped(p, bm, bn)) continue;
        int kb0, kb1;
        k_range(p, bm, bn, nkb, kb0, kb1);
        // one TMEM accumulation per CHUNK_KB k-slices (CHUNK_KB * 32 of K)
        for (int kc = kb0; kc < kb1 && ok; kc += CHUNK_KB) {
          if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
          const int kend = min(kb1, kc + CHUNK_KB);
          for (int kb = kc; kb < kend; ++kb) {
            if (!mbar_wait(&conv[stage], phase, abort_flag)) {
              ok = false;
              break;
            }
            fence_after();
            const uint32_t bh = smem_u32(b_hi(stage)), bl = smem_u32(b_lo(stage));
            const uint32_t a_hi_t = tmem_base + (uint32_t)(A_TMEM_COL0 + stage * 2 * BK);
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk) {
              // B: K-major SW128, 8 tf32 = 32 bytes per k-step inside each 128-byte row;
              // A: 8 TMEM columns per k-step
              const uint64_t dbh = make_desc(bh + kk * 32, 16, 1024);
              const uint64_t dbl = make_desc(bl + kk * 32, 16, 1024);
              const uint32_t ah = a_hi_t + kk * 8, al = a_hi_t + BK + kk * 8;
              const uint32_t first = (kb == kc && kk == 0) ? 0u : 1u;
              umma_tf32_ts(d_tmem, al, dbh, id, first);
              umma_tf32_ts(d_tmem, ah, dbl, id, 1u);
              umma_tf32_ts(d_tmem, ah, dbh, id, 1u);
            }
            umma_commit(&empty[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          umma_commit(&tfull[acc]);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
      }
    }
  } else if (warp < 6) {
    // converters: A row `arow` (this warp's TMEM lane quarter) split into hi and
    // lo straight into TMEM; B lo = raw - hi into shared memory (the raw B tile
    // itself serves as B hi: kind::tf32 ignores the low 13 bits)
    const int ct = threadIdx.x - 64;  // 0..127
    const int quarter = warp & 3;
    const int arow = quarter * 32 + lane;
    const uint32_t a_lane = (uint32_t)(quarter * 32) << 16;
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x) {
      const int bm = t % p.mb, bn = t / p.mb;
      if (tile_skipped(p, bm, bn)) continue;
      int kb0, kb1;
      k_range(p, bm, bn, nkb, kb0, kb1);
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag)) {
          ok = false;
          break;
        }
        {
          // row arow of the SW128 K-major A tile: 16-byte chunk c sits at c ^ (row % 8)
          const uint8_t* rowp = a_raw(stage) + arow * 128;
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 x = *reinterpret_cast<const uint4*>(rowp + ((c ^ (arow & 7)) << 4));
            const uint32_t v[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              hi[4 * c + e] = v[e] & 0xFFFFE000u;
              lo[4 * c + e] = __float_as_uint(__uint_as_float(v[e]) - __uint_as_float(hi[4 * c + e]));
            }
          }
          const uint32_t tcol = tmem_base + a_lane + (uint32_t)(A_TMEM_COL0 + stage * 2 * BK);
          tmem_st32(tcol, hi);
          tmem_st32(tcol + BK, lo);
        }
        uint4* bh4 = reinterpret_cast<uint4*>(b_hi(stage));
        uint4* bl4 = reinterpret_cast<uint4*>(b_lo(stage));
#pragma unroll 4
        for (int i = ct; i < B_BYTES / 16; i += 128) {
          const uint4 x = bh4[i];
          bl4[i] = lo_part(x);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        fence_before();
        mbar_arrive(&conv[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
    }
  } else {
    // epilogue warps 6..9
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < p.num_tiles && !*abort_flag; t += gridDim.x) {
      const int bm = t % p.mb, bn = t / p.mb;
      if (tile_skipped(p, bm, bn)) continue;
      // chunk results summed in fp32 registers (round-to-nearest adds)
      float sum[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) sum[j] = 0.f;
      int kb0, kb1;
      k_range(p, bm, bn, nkb, kb0, kb1);
      for (int kc = kb0; kc < kb1; kc += CHUNK_KB) {
        if (!mbar_wait(&tfull[acc], acc_phase, abort_flag)) {
          ok = false;
          break;
        }
        fence_after();
#pragma unroll
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint32_t r[32];
          tmem_ld32(tmem_base + lane_addr + (uint32_t)(acc * BN + cc * 32), r);
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[cc * 32 + j] += __uint_as_float(r[j]);
        }
        fence_before();
        mbar_arrive(&tempty[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) break;
      const int64_t row = (int64_t)bm * BM + row_in_tile;
      const int64_t col0 = (int64_t)bn * BN;
      if (p.c_mode != 0) {
        // 32-column chunks staged in shared memory and written by the tensor
        // engine: a plain store (beta 0) or an fp32 add into C at L2 (beta 1,
        // C + alpha * sum rounded once, as fmaf(1, C, alpha * sum) would be).
        // Rows and columns past M, N are clipped by the tensor map.
#pragma unroll
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint8_t* buf = c_stage + (quarter * 2 + (cc & 1)) * C_CHUNK_BYTES;
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          __syncwarp();
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 v = make_float4(p.alpha * sum[cc * 32 + 4 * j4], p.alpha * sum[cc * 32 + 4 * j4 + 1],
                                         p.alpha * sum[cc * 32 + 4 * j4 + 2],
                                         p.alpha * sum[cc * 32 + 4 * j4 + 3]);
            *reinterpret_cast<float4*>(buf + lane * 128 + ((j4 ^ (lane & 7)) << 4)) = v;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            const int x = (int)(col0 + cc * 32), y = (int)(bm * BM + quarter * 32);
            if (p.c_mode == 2)
              asm volatile(
                  "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group"
                  " [%0, {%2, %3}], [%1];" ::"l"(reinterpret_cast<uint64_t>(&map_c)),
                  "r"(smem_u32(buf)), "r"(x), "r"(y)
                  : "memory");
            else
              asm volatile(
                  "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group"
                  " [%0, {%2, %3}], [%1];" ::"l"(reinterpret_cast<uint64_t>(&map_c)),
                  "r"(smem_u32(buf)), "r"(x), "r"(y)
                  : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
        }
      } else if (row < p.M) {
        float* cp = p.c + row * p.ldc + col0;
        const bool vec = (col0 + BN <= p.N) && ((reinterpret_cast<uintptr_t>(cp) & 15) == 0);
        if (vec) {
#pragma unroll
          for (int j = 0; j < BN; j += 4) {
            float4 v = make_float4(p.alpha * sum[j], p.alpha * sum[j + 1], p.alpha * sum[j + 2],
                                   p.alpha * sum[j + 3]);
            if (p.beta != 0.f) {
              float4 o = *reinterpret_cast<const float4*>(cp + j);
              v.x = fmaf(p.beta, o.x, v.x);
              v.y = fmaf(p.beta, o.y, v.y);
              v.z = fmaf(p.beta, o.z, v.z);
              v.w = fmaf(p.beta, o.w, v.w);
            }
            *reinterpret_cast<float4*>(cp + j) = v;
          }
        } else {
#pragma unroll
          for (int j = 0; j < BN; ++j) {
            if (col0 + j < p.N) {
              float v = p.alpha * sum[j];
              if (p.beta != 0.f) v = fmaf(p.beta, cp[j], v);
              cp[j] = v;
            }
          }
        }
      }
    }
  }

  // tensor stores must finish (shared memory read, global writes done) before exit
  if (warp >= 6 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS));
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// fp32 [rows, cols] row-major map (ld elements) with box {32 inner, box_rows}.
static int make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(GQ_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 4)};
  cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GQ_ECUDA, "cuTensorMapEncodeTiled(fp32) failed (%d)", (int)r);
  return GQ_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// True when the tensor-core path accepts the problem.
bool eligible(int ta, int tb, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
              const float* B, int64_t ldb, const float* C, int64_t ldc) {
  (void)C;
  (void)ldc;
  // Both operands K-major only: for 32-bit MN-major operands the UMMA wants the
  // 32-byte-atom 128B swizzle, which this kernel's TMA loads do not produce.
  if (ta != 0 || tb != 1) return false;
  // M may be anything >= 1 (rows past M are zero-filled by TMA and not
  // stored), so the arithmetic a row gets does not depend on how many rows
  // share the call; N and K are fixed by the operands' shapes.
  if (M < 1 || N < 128 || K < 32) return false;
  if (!aligned16(A) || !aligned16(B)) return false;
  if ((lda & 3) || (ldb & 3)) return false;
  if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) return false;
  return true;
}

int launch(int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
           const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int uplo, int tri,
           cudaStream_t st) {
  CUtensorMap ma, mbm;
  GQ_TRY(make_map(&ma, A, M, K, lda, BM));
  if (tb) GQ_TRY(make_map(&mbm, B, N, K, ldb, BN));
  else GQ_TRY(make_map(&mbm, B, K, N, ldb, BK));
  Params p;
  p.c = C;
  p.ldc = ldc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.alpha = alpha;
  p.beta = beta;
  p.uplo = uplo;
  p.tri = tri;
  p.mb = (int)ceil_div(M, BM);
  p.nb = (int)ceil_div(N, BN);
  p.num_tiles = p.mb * p.nb;
  p.b_kmajor = tb;
  CUtensorMap mc = ma;  // unused unless c_mode != 0
  p.c_mode = 0;
  if ((beta == 0.f || beta == 1.f) && aligned16(C) && (ldc & 3) == 0 && ldc >= N) {
    GQ_TRY(make_map(&mc, C, M, N, ldc, 32));
    p.c_mode = (beta == 0.f) ? 1 : 2;
  }
  static int attr_device = -1;
  int dev = 0;
  GQ_CHECK_CUDA(cudaGetDevice(&dev));
  if (attr_device != dev) {
    GQ_CHECK_CUDA(cudaFuncSetAttribute(tf32x3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_BYTES));
    attr_device = dev;
  }
  const int grid = std::min(p.num_tiles, cta_budget());
  tf32x3_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(ma, mbm, mc, p);
  return check_launch("tcgen05 tf32x3 gemm");
}

// Failure-path check of this file's bounded wait: one thread waits on an
// mbarrier that nothing arrives on, so mbar_wait must give up after
// g_wait_limit_ns, record GQ_DEVERR_TIMEOUT and return false; *observed gets
// 1 when it did.  No trap, no fault: the kernel then simply returns.
__global__ void expire_wait_kernel(int* observed) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) *observed = mbar_wait(&bar, 0, &abort_flag) ? 0 : 1;
}

int set_wait_limit(uint64_t ns) {
  GQ_CHECK_CUDA(cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns)));
  return GQ_OK;
}

int launch_expire_test(int* observed, cudaStream_t st) {
  expire_wait_kernel<<<1, 32, 0, st>>>(observed);
  return check_launch("tf32x3 expire_wait");
}

}  // namespace tc32
}  // namespace gq

extern "C" int gq_gemm_f32_tc(int trans_b, int64_t M, int64_t N, int64_t K, float alpha,
                              const float* a, int64_t lda, const float* b, int64_t ldb, float beta,
                              float* c, int64_t ldc, int uplo, void* stream) {
  GQ_REQUIRE(gq::tc32::eligible(0, trans_b, M, N, K, a, lda, b, ldb, c, ldc),
             "gq_gemm_f32_tc: needs M >= 1, N >= 128, K >= 32, 16-byte aligned operands and leading "
             "dimensions that are multiples of 4");
  GQ_REQUIRE(uplo >= 0 && uplo <= 2, "gq_gemm_f32_tc: bad uplo");
  return gq::tc32::launch(trans_b ? 1 : 0, M, N, K, alpha, a, lda, b, ldb, beta, c, ldc, uplo, 0,
                          gq::as_stream(stream));
}
