// Activation statistics on the tcgen05 tensor cores (stats.py:16-17):
//   C[M, N] (+)= A^T B   with A = xa [K, M], B = xb [K, N] (bf16, row-major,
//   K = tokens), fp32 accumulation in tensor memory.
//
// Both operands are read in their native [tokens, features] layout: a TMA
// box of 64 features x 64 tokens with 128-byte swizzle is exactly one
// MN-major SW128 canonical block for the UMMA descriptor, so no transpose
// pass is needed.  Two forms compute the same bits:
//   pair (default): clusters of two CTAs, one 256 x 256 tile per cluster,
//     tcgen05 cta_group::2 MMAs (M256 N256 K16) issued by the even CTA over
//     both CTAs' shared memory; each CTA stages only its half of A and of B
//     (32 KB per 64-token stage, six stages);
//   single: one CTA per SM, tiles of 128 x 256 (48 KB per stage, four
//     stages), used where no cluster of two fits.
// In both, per CTA:
//   warp 0      TMA producer (one thread);
//   warp 1      MMA issuer (one thread; in the pair form only the even CTA's),
//               restarting the accumulation every CHUNK_KB stages (1024
//               tokens), two TMEM accumulators of 256 columns;
//   warps 2-9   epilogue: add each chunk's TMEM result into fp32 registers
//               (128 columns per thread) and store the tile once; when
//               accumulating, the register sum starts from C's contents.
// Summing 1024-token chunks outside the tensor core keeps H within 1e-5 of a
// float64 reference over hundreds of thousands of tokens (3.0e-6 worst
// normalized element at 262,144 tokens, d = 11008); a single TMEM
// accumulation over 4096 tokens already drifts past that bound.
// For the symmetric case (xa == xb) only tiles touching the upper triangle
// are computed and the result is mirrored afterwards.
//
// Every mbarrier wait is bounded by a globaltimer deadline; a wait that
// expires raises a shared abort flag (all roles leave their loops) and
// records GQ_DEVERR_TIMEOUT in the device status word read by
// gq_device_status().  No load uses multicast, so the kernels are safe on
// any number of GPUs.
#include <cuda.h>

#include "gq_common.cuh"

namespace gq {

__device__ int g_device_status = 0;
// this file's bound on every mbarrier wait (gq_set_wait_limit_ns)
static __device__ uint64_t g_wait_limit_ns = kWaitLimitNs;

namespace tc {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_STAGE = BM * BK * 2;       // 16 KB
constexpr int B_STAGE = BN * BK * 2;       // 32 KB
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int BOX_BYTES = 64 * BK * 2;     // one 64-feature x 64-token box: 8 KB
constexpr int TMEM_COLS = 512;
constexpr int THREADS = 320;       // TMA warp, MMA warp, 8 epilogue warps
constexpr int EPI_THREADS = 256;
constexpr int HALF_COLS = BN / 2;  // accumulator columns per epilogue thread
constexpr int CHUNK_KB = 16;       // k-blocks (x 64 tokens) per TMEM accumulation
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

// kind::f16 instruction descriptor: D f32, A/B bf16, both MN-major, N=256, M=128.
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
                           ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

struct Params {
  float* c;
  int64_t ldc;
  int64_t M, N, K;
  int symmetric;
  int accumulate;
  int num_tiles;
  int mb;  // row tiles
  int nb;  // column tiles
  int diag_only;  // symmetric: only the tiles holding diagonal elements
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
// Bounded wait; false when the deadline passed or another role aborted.
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

// SW128 UMMA shared-memory descriptor (sm100 format, version 1).
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for tcgen05
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accum));
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

// Rows of column tile bn that are computed: all of them, or for the
// symmetric case the row tiles 0 .. min(mb, 2 bn + 2) - 1 touching the upper
// triangle (non-decreasing in bn).
__device__ __forceinline__ int col_height(const Params& p, int bn) {
  return p.symmetric ? min(p.mb, 2 * bn + 2) : p.mb;
}

// Tile index -> (row tile, column tile).  Tiles are taken in groups of
// GROUP_COLS column tiles and, inside a group, row by row, so the CTAs that
// stream the same token slabs at the same time share about GROUP_COLS column
// panels and grid / GROUP_COLS row panels of the operands: each wave of tiles
// reads under half of X from DRAM and L2 serves the rest.
constexpr int GROUP_COLS = 8;
__device__ __forceinline__ void tile_coords(const Params& p, int t, int& bm, int& bn) {
  if (p.diag_only) {  // 128-row tile t holds its diagonal in 256-column tile t / 2
    bm = t;
    bn = t >> 1;
    return;
  }
  for (int g0 = 0; g0 < p.nb; g0 += GROUP_COLS) {
    const int g1 = min(p.nb, g0 + GROUP_COLS);
    int cnt = 0;
    for (int j = g0; j < g1; ++j) cnt += col_height(p, j);
    if (t >= cnt) {
      t -= cnt;
      continue;
    }
    // row r of the group holds the columns whose height exceeds r: a suffix
    int first = g0;
    for (int r = 0; r < col_height(p, g1 - 1); ++r) {
      while (first < g1 && col_height(p, first) <= r) ++first;
      const int n = g1 - first;
      if (t < n) {
        bm = r;
        bn = first + t;
        return;
      }
      t -= n;
    }
  }
  bm = 0;
  bn = 0;
}

__global__ void __launch_bounds__(THREADS, 1)
gemm_tn_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * A_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + STAGES * B_STAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // epilogue: warp 2's outcome of each accumulator wait, by chunk parity
  volatile int* epi_go = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_THREADS);
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
        int bm, bn;
        tile_coords(p, t, bm, bn);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
          mbar_expect_tx(&full[stage], STAGE_BYTES);
          const int k0 = kb * BK;
          uint8_t* a_dst = sa + stage * A_STAGE;
          uint8_t* b_dst = sb + stage * B_STAGE;
          tma_load_2d(&map_a, &full[stage], a_dst, bm * BM, k0);
          tma_load_2d(&map_a, &full[stage], a_dst + BOX_BYTES, bm * BM + 64, k0);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            tma_load_2d(&map_b, &full[stage], b_dst + q * BOX_BYTES, bn * BN + q * 64, k0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles && !*abort_flag; t += gridDim.x) {
        // one TMEM accumulation per chunk of CHUNK_KB k-blocks (CHUNK_KB * 64 tokens)
        for (int kc = 0; kc < nkb && ok; kc += CHUNK_KB) {
          if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
          const int kend = min(nkb, kc + CHUNK_KB);
          for (int kb = kc; kb < kend; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag)) {
              ok = false;
              break;
            }
            fence_after();
            const uint32_t a_base = smem_u32(sa + stage * A_STAGE);
            const uint32_t b_base = smem_u32(sb + stage * B_STAGE);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              // 16 tokens = 16 rows of 128 B; M/N chunks of 64 features are BOX_BYTES
              // apart, groups of 8 token rows are 1024 B apart.
              const uint64_t ad = make_desc(a_base + kk * 2048, BOX_BYTES, 1024);
              const uint64_t bd = make_desc(b_base + kk * 2048, BOX_BYTES, 1024);
              umma_bf16(d_tmem, ad, bd, (kb > kc || kk > 0) ? 1u : 0u);
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
  } else {
    // epilogue warps 2..9: warp w may access TMEM lanes 32*(w%4) .. +31; warps 2-5
    // take accumulator columns 0-127, warps 6-9 columns 128-255.  Chunk results
    // are summed in fp32 registers (round-to-nearest adds), so each TMEM
    // accumulation spans only CHUNK_KB * 64 tokens.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    uint32_t chunk = 0;
    // Only warp 2 polls the accumulator barrier; the other epilogue warps
    // sleep at a named barrier instead of spinning (their issue slots belong
    // to the MMA and TMA threads on the same schedulers).  Control flow stays
    // uniform across the eight warps: every loop decision uses warp 2's
    // outcome, published before the named barrier.
    for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
      int bm, bn;
      tile_coords(p, t, bm, bn);
      const int64_t row = (int64_t)bm * BM + row_in_tile;
      const int64_t col0 = (int64_t)bn * BN + half * HALF_COLS;
      const bool inside = row < p.M && col0 < p.N;
      float* cp = p.c + row * p.ldc + col0;
      const bool vec = inside && (col0 + HALF_COLS <= p.N) &&
                       ((reinterpret_cast<uintptr_t>(cp) & 15) == 0);
      // the running sum starts from C when accumulating, so a product split
      // into launches at multiples of CHUNK_KB * BK tokens adds the same
      // chunk results in the same order as one launch over all tokens
      float sum[HALF_COLS];
      if (p.accumulate && vec) {
#pragma unroll
        for (int j = 0; j < HALF_COLS; j += 4) {
          const float4 o = *reinterpret_cast<const float4*>(cp + j);
          sum[j] = o.x;
          sum[j + 1] = o.y;
          sum[j + 2] = o.z;
          sum[j + 3] = o.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < HALF_COLS; ++j)
          sum[j] = (p.accumulate && inside && col0 + j < p.N) ? cp[j] : 0.f;
      }
      for (int kc = 0; kc < nkb; kc += CHUNK_KB) {
        if (warp == 2) {
          const bool got = mbar_wait(&tfull[acc], acc_phase, abort_flag);
          if (lane == 0) epi_go[chunk & 1] = got ? 1 : 0;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(EPI_THREADS) : "memory");
        ok = epi_go[chunk & 1] != 0;
        ++chunk;
        if (!ok) break;
        fence_after();
#pragma unroll
        for (int c = 0; c < HALF_COLS / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem_base + lane_addr + (uint32_t)(acc * BN + half * HALF_COLS + c * 32), r);
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[c * 32 + j] += __uint_as_float(r[j]);
        }
        fence_before();
        mbar_arrive(&tempty[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) break;
      if (vec) {
#pragma unroll
        for (int j = 0; j < HALF_COLS; j += 4)
          *reinterpret_cast<float4*>(cp + j) = make_float4(sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
      } else if (inside) {
#pragma unroll
        for (int j = 0; j < HALF_COLS; ++j)
          if (col0 + j < p.N) cp[j] = sum[j];
      }
    }
  }

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

// [tokens, features] bf16 map with a 64 x 64 box, 128-byte swizzle.
static int make_map(CUtensorMap* map, const void* x, int64_t tokens, int64_t feats, int64_t ld) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(GQ_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)feats, (cuuint64_t)tokens};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)BK};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GQ_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return GQ_OK;
}

static int check_operand(const char* who, const void* x, int64_t tokens, int64_t feats,
                         int64_t ld) {
  GQ_REQUIRE(x != nullptr, "%s: NULL activations", who);
  GQ_REQUIRE(tokens >= 0 && feats > 0 && ld >= feats, "%s: bad shape", who);
  GQ_REQUIRE(ld % 8 == 0, "%s: ld must be a multiple of 8 elements (16-byte TMA stride)", who);
  GQ_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0, "%s: activations must be 16-byte aligned",
             who);
  GQ_REQUIRE(tokens < (1ll << 31) && feats < (1ll << 31), "%s: dimension too large", who);
  return GQ_OK;
}

int launch_single(const void* xa, int64_t lda, const void* xb, int64_t ldb, int64_t K, int64_t M,
                  int64_t N, float* c, int64_t ldc, int accumulate, int symmetric, cudaStream_t st,
                  int diag_only) {
  if (K == 0) {
    if (!accumulate)
      GQ_CHECK_CUDA(cudaMemset2DAsync(c, ldc * 4, 0, N * 4, M, st));
    return GQ_OK;
  }
  CUtensorMap ma, mbm;
  GQ_TRY(make_map(&ma, xa, K, M, lda));
  GQ_TRY(make_map(&mbm, xb, K, N, ldb));
  Params p;
  p.c = c;
  p.ldc = ldc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.symmetric = symmetric;
  p.accumulate = accumulate;
  p.mb = (int)ceil_div(M, BM);
  p.nb = (int)ceil_div(N, BN);
  p.diag_only = symmetric && diag_only;
  if (p.diag_only) {
    p.num_tiles = p.mb;
  } else if (symmetric) {
    int64_t cnt = 0;
    for (int j = 0; j < p.nb; ++j) cnt += std::min(p.mb, 2 * j + 2);
    p.num_tiles = (int)cnt;
  } else {
    p.num_tiles = p.mb * p.nb;
  }
  static int attr_device = -1;
  int dev = 0;
  GQ_CHECK_CUDA(cudaGetDevice(&dev));
  if (attr_device != dev) {
    GQ_CHECK_CUDA(cudaFuncSetAttribute(gemm_tn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       SMEM_BYTES));
    attr_device = dev;
  }
  const int grid = std::min(p.num_tiles, cta_budget());
  gemm_tn_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(ma, mbm, p);
  return check_launch("tcgen05 gemm_tn");
}

}  // namespace tc

// ---------------------------------------------------------------------------
// CTA-pair form (tcgen05 cta_group::2): one cluster of two CTAs computes a
// 256 x 256 tile.  CTA r of the pair loads rows [128 r, 128 r + 128) of the
// tile's A panel and columns [128 r, 128 r + 128) of its B panel (32 KB per
// 64-token stage instead of 48 KB), and each CTA's tensor memory holds its
// 128 rows x 256 columns of the accumulator.  The even CTA issues the MMAs
// (M = 256, N = 256, K = 16), which read both CTAs' shared memory at the same
// offsets.  Protocol:
//   full[s]   (even CTA): its producer's expect_tx for both halves; both
//             producers' TMA loads complete_tx on it;
//   empty[s]  (each CTA): one arrival from the MMA thread's commit, so each
//             producer may refill its half of the stage;
//   tfull[a]  (each CTA): committed by the MMA thread after a chunk;
//   tempty[a] (even CTA): one arrival per epilogue warp of both CTAs.
// Loads use no multicast; the even CTA's barriers are reached through mapa
// addresses.  The arithmetic per element (1024-token chunks summed in fp32
// registers, in token order) is the one-CTA kernel's.
namespace tc2 {
using namespace tc;

constexpr int PM = 256;   // tile rows (128 per CTA)
constexpr int HM = 128;
constexpr int PN = 256;   // tile columns (128 loaded per CTA)
constexpr int STAGES2 = 6;
constexpr int HALF_STAGE = 2 * BOX_BYTES;   // 128 features x 64 tokens
constexpr int STAGE2 = 2 * HALF_STAGE;      // A half + B half
constexpr int EPI_WARPS = EPI_THREADS / 32;
constexpr int SMEM2 = STAGES2 * STAGE2 + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t IDESC2 = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
                            ((uint32_t)(PN >> 3) << 17) | ((uint32_t)(PM >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tma_load_pair(const CUtensorMap* map, uint32_t bar_cluster,
                                              void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                               uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(IDESC2), "r"(accum));
}
// one arrival on the barrier at this shared-memory offset in both CTAs of the
// pair once this thread's earlier MMAs are complete (a commit, not a load)
__device__ __forceinline__ void umma_commit_both(const uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}
__device__ __forceinline__ void remote_arrive(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}

// Column tile bn computes row tiles 0 .. col_height2 - 1 (256 rows each).
__device__ __forceinline__ int col_height2(const Params& p, int bn) {
  return p.symmetric ? min(p.mb, bn + 1) : p.mb;
}
// Same grouped order as the one-CTA kernel, in 256 x 256 tiles.
__device__ __forceinline__ void tile_coords2(const Params& p, int t, int& bm, int& bn) {
  if (p.diag_only) {
    bm = bn = t;
    return;
  }
  for (int g0 = 0; g0 < p.nb; g0 += GROUP_COLS) {
    const int g1 = min(p.nb, g0 + GROUP_COLS);
    int cnt = 0;
    for (int j = g0; j < g1; ++j) cnt += col_height2(p, j);
    if (t >= cnt) {
      t -= cnt;
      continue;
    }
    int first = g0;
    for (int r = 0; r < col_height2(p, g1 - 1); ++r) {
      while (first < g1 && col_height2(p, first) <= r) ++first;
      const int n = g1 - first;
      if (t < n) {
        bm = r;
        bn = first + t;
        return;
      }
      t -= n;
    }
  }
  bm = 0;
  bn = 0;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
gemm_tn_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                    const __grid_constant__ CUtensorMap map_b, Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES2 * STAGE2);
  uint64_t* empty = full + STAGES2;
  uint64_t* tfull = empty + STAGES2;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* epi_go = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int cid = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
  }
  if (warp == 1) {
    // collective over the pair: warp 1 of both CTAs, same destination offset
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  fence_before();
  cluster_sync();  // barriers initialised and the allocation visible in both CTAs
  fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nkb = (int)((p.K + BK - 1) / BK);
  const uint32_t full0 = peer_addr(&full[0], 0);      // the even CTA's barriers
  const uint32_t tempty0 = peer_addr(&tempty[0], 0);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = cid; t < p.num_tiles && !*abort_flag; t += nclusters) {
        int bm, bn;
        tile_coords2(p, t, bm, bn);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
          if (leader) mbar_expect_tx(&full[stage], 2 * STAGE2);
          const int k0 = kb * BK;
          uint8_t* a_dst = smem + stage * STAGE2;
          uint8_t* b_dst = a_dst + HALF_STAGE;
          const uint32_t bar = full0 + 8u * (uint32_t)stage;
          const int r0 = bm * PM + (int)rank * HM, c0 = bn * PN + (int)rank * HM;
          tma_load_pair(&map_a, bar, a_dst, r0, k0);
          tma_load_pair(&map_a, bar, a_dst + BOX_BYTES, r0 + 64, k0);
          tma_load_pair(&map_b, bar, b_dst, c0, k0);
          tma_load_pair(&map_b, bar, b_dst + BOX_BYTES, c0 + 64, k0);
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // every stage released by the MMA: no commit arrival is still on its
      // way to this CTA's barriers when the pair tears down
      for (int i = 0; i < STAGES2 && !*abort_flag; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
        if (++stage == STAGES2) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = cid; ok && t < p.num_tiles && !*abort_flag; t += nclusters) {
        for (int kc = 0; kc < nkb && ok; kc += CHUNK_KB) {
          if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(acc * PN);
          const int kend = min(nkb, kc + CHUNK_KB);
          for (int kb = kc; kb < kend; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag)) {
              ok = false;
              break;
            }
            fence_after();
            const uint32_t a_base = smem_u32(smem + stage * STAGE2);
            const uint32_t b_base = a_base + HALF_STAGE;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint64_t ad = make_desc(a_base + kk * 2048, BOX_BYTES, 1024);
              const uint64_t bd = make_desc(b_base + kk * 2048, BOX_BYTES, 1024);
              umma_bf16_pair(d_tmem, ad, bd, (kb > kc || kk > 0) ? 1u : 0u);
            }
            umma_commit_both(&empty[stage]);
            if (++stage == STAGES2) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          umma_commit_both(&tfull[acc]);
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1;
          }
        }
      }
    }
  } else {
    // epilogue warps 2..9 of each CTA: this CTA's 128 rows, 256 columns
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    uint32_t chunk = 0;
    for (int t = cid; ok && t < p.num_tiles; t += nclusters) {
      int bm, bn;
      tile_coords2(p, t, bm, bn);
      const int64_t row = (int64_t)bm * PM + (int64_t)rank * HM + row_in_tile;
      const int64_t col0 = (int64_t)bn * PN + half * HALF_COLS;
      const bool inside = row < p.M && col0 < p.N;
      float* cp = p.c + row * p.ldc + col0;
      const bool vec = inside && (col0 + HALF_COLS <= p.N) &&
                       ((reinterpret_cast<uintptr_t>(cp) & 15) == 0);
      float sum[HALF_COLS];
      if (p.accumulate && vec) {
#pragma unroll
        for (int j = 0; j < HALF_COLS; j += 4) {
          const float4 o = *reinterpret_cast<const float4*>(cp + j);
          sum[j] = o.x;
          sum[j + 1] = o.y;
          sum[j + 2] = o.z;
          sum[j + 3] = o.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < HALF_COLS; ++j)
          sum[j] = (p.accumulate && inside && col0 + j < p.N) ? cp[j] : 0.f;
      }
      for (int kc = 0; kc < nkb; kc += CHUNK_KB) {
        if (warp == 2) {
          const bool got = mbar_wait(&tfull[acc], acc_phase, abort_flag);
          if (lane == 0) epi_go[chunk & 1] = got ? 1 : 0;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(EPI_THREADS) : "memory");
        ok = epi_go[chunk & 1] != 0;
        ++chunk;
        if (!ok) break;
        fence_after();
#pragma unroll
        for (int c = 0; c < HALF_COLS / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem_base + lane_addr + (uint32_t)(acc * PN + half * HALF_COLS + c * 32), r);
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[c * 32 + j] += __uint_as_float(r[j]);
        }
        fence_before();
        __syncwarp();
        if (lane == 0) remote_arrive(tempty0 + 8u * (uint32_t)acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) break;
      if (vec) {
#pragma unroll
        for (int j = 0; j < HALF_COLS; j += 4)
          *reinterpret_cast<float4*>(cp + j) = make_float4(sum[j], sum[j + 1], sum[j + 2], sum[j + 3]);
      } else if (inside) {
#pragma unroll
        for (int j = 0; j < HALF_COLS; ++j)
          if (col0 + j < p.N) cp[j] = sum[j];
      }
    }
  }

  // both CTAs done with the pair's shared memory and tensor memory
  fence_before();
  cluster_sync();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS));
  }
  cluster_sync();
}


int pair_setup(int* max_clusters) {
  static int attr_device = -1, clusters = 0;
  int dev = 0;
  GQ_CHECK_CUDA(cudaGetDevice(&dev));
  if (attr_device != dev) {
    GQ_CHECK_CUDA(cudaFuncSetAttribute(gemm_tn_pair_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM2;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    GQ_CHECK_CUDA(cudaOccupancyMaxActiveClusters(&clusters, gemm_tn_pair_kernel, &cfg));
    GQ_REQUIRE(clusters >= 1, "tcgen05 pair kernel: no cluster of two CTAs fits on this device");
    attr_device = dev;
  }
  *max_clusters = clusters;
  return GQ_OK;
}

// C (+)= A^T B with CTA pairs; same contract as tc::launch.
int launch_pair(const void* xa, int64_t lda, const void* xb, int64_t ldb, int64_t K, int64_t M,
                int64_t N, float* c, int64_t ldc, int accumulate, int symmetric, cudaStream_t st,
                int diag_only) {
  if (K == 0) {
    if (!accumulate) GQ_CHECK_CUDA(cudaMemset2DAsync(c, ldc * 4, 0, N * 4, M, st));
    return GQ_OK;
  }
  CUtensorMap ma, mbm;
  GQ_TRY(make_map(&ma, xa, K, M, lda));
  GQ_TRY(make_map(&mbm, xb, K, N, ldb));
  Params p;
  p.c = c;
  p.ldc = ldc;
  p.M = M;
  p.N = N;
  p.K = K;
  p.symmetric = symmetric;
  p.accumulate = accumulate;
  p.mb = (int)ceil_div(M, PM);
  p.nb = (int)ceil_div(N, PN);
  p.diag_only = symmetric && diag_only;
  if (p.diag_only) {
    p.num_tiles = std::min(p.mb, p.nb);
  } else if (symmetric) {
    int64_t cnt = 0;
    for (int j = 0; j < p.nb; ++j) cnt += std::min(p.mb, j + 1);
    p.num_tiles = (int)cnt;
  } else {
    p.num_tiles = p.mb * p.nb;
  }
  int max_clusters = 0;
  GQ_TRY(pair_setup(&max_clusters));
  const int clusters = std::max(1, std::min(std::min(p.num_tiles, cta_budget() / 2), max_clusters));
  gemm_tn_pair_kernel<<<2 * clusters, THREADS, SMEM2, st>>>(ma, mbm, p);
  return check_launch("tcgen05 gemm_tn pair");
}

}  // namespace tc2

namespace tc {
// CTA pairs where a cluster of two fits (bit-identical results), else one CTA
// per tile.  diag_only (symmetric): only the tiles that hold diagonal
// elements, each computed exactly as in the full launch.
int launch(const void* xa, int64_t lda, const void* xb, int64_t ldb, int64_t K, int64_t M,
           int64_t N, float* c, int64_t ldc, int accumulate, int symmetric, cudaStream_t st,
           int diag_only) {
  int max_clusters = 0;
  if (pair_kernels() && tc2::pair_setup(&max_clusters) == GQ_OK && max_clusters >= 1)
    return tc2::launch_pair(xa, lda, xb, ldb, K, M, N, c, ldc, accumulate, symmetric, st,
                            diag_only);
  (void)cudaGetLastError();  // the failed occupancy query is not this launch's error
  return launch_single(xa, lda, xb, ldb, K, M, N, c, ldc, accumulate, symmetric, st, diag_only);
}
}  // namespace tc

int symmetrize_upper(float* h, int64_t d, int64_t ldh, cudaStream_t st);

namespace tc {
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
}  // namespace tc

namespace tc32 {
int read_status(int reset, int* out);
int set_wait_limit(uint64_t ns);
int launch_expire_test(int* observed, cudaStream_t st);
}

}  // namespace gq

extern "C" {

int gq_syrk_bf16(const uint16_t* x, int64_t tokens, int64_t d, int64_t ldx, float* h, int64_t ldh,
                 int accumulate, void* stream) {
  GQ_TRY(gq::tc::check_operand("gq_syrk_bf16", x, tokens, d, ldx));
  GQ_REQUIRE(h != nullptr && ldh >= d, "gq_syrk_bf16: bad output");
  cudaStream_t st = gq::as_stream(stream);
  GQ_TRY(gq::tc::launch(x, ldx, x, ldx, tokens, d, d, h, ldh, accumulate, 1, st, 0));
  return gq::symmetrize_upper(h, d, ldh, st);
}

int gq_gemm_tn_bf16(const uint16_t* xa, int64_t lda, const uint16_t* xb, int64_t ldb,
                    int64_t tokens, int64_t da, int64_t db, float* g, int64_t ldg, int accumulate,
                    void* stream) {
  GQ_TRY(gq::tc::check_operand("gq_gemm_tn_bf16", xa, tokens, da, lda));
  GQ_TRY(gq::tc::check_operand("gq_gemm_tn_bf16", xb, tokens, db, ldb));
  GQ_REQUIRE(g != nullptr && ldg >= db, "gq_gemm_tn_bf16: bad output");
  return gq::tc::launch(xa, lda, xb, ldb, tokens, da, db, g, ldg, accumulate, 0,
                        gq::as_stream(stream), 0);
}

int gq_set_wait_limit_ns(uint64_t ns) {
  GQ_REQUIRE(ns >= 1000000ull && ns <= 60000000000ull,
             "gq_set_wait_limit_ns: %llu ns is outside [1 ms, 60 s]", (unsigned long long)ns);
  GQ_TRY(gq::tc::set_wait_limit(ns));
  return gq::tc32::set_wait_limit(ns);
}

int gq_test_expire_wait(int unit, int* observed, void* stream) {
  GQ_REQUIRE(observed != nullptr, "gq_test_expire_wait: NULL observed");
  GQ_REQUIRE(unit == 0 || unit == 1, "gq_test_expire_wait: unit must be 0 or 1");
  if (unit == 1) return gq::tc32::launch_expire_test(observed, gq::as_stream(stream));
  gq::tc::expire_wait_kernel<<<1, 32, 0, gq::as_stream(stream)>>>(observed);
  return gq::check_launch("bf16 expire_wait");
}

int gq_check_device(void* stream) {
  int v = 0;
  GQ_TRY(gq_device_status(&v, 1, stream));
  if (v == gq::GQ_DEVERR_TIMEOUT)
    return gq::fail(GQ_ETIMEOUT, "a bounded device-side wait expired: a kernel gave up and "
                                 "returned early, so its outputs are incomplete");
  if (v != gq::GQ_DEVERR_NONE) return gq::fail(GQ_ECUDA, "device status word %d", v);
  return GQ_OK;
}

int gq_device_status(int* status_out, int reset, void* stream) {
  GQ_REQUIRE(status_out != nullptr, "gq_device_status: NULL output");
  cudaStream_t st = gq::as_stream(stream);
  GQ_CHECK_CUDA(cudaStreamSynchronize(st));
  int v = 0;
  GQ_CHECK_CUDA(cudaMemcpyFromSymbol(&v, gq::g_device_status, sizeof(int)));
  if (reset) {
    int z = 0;
    GQ_CHECK_CUDA(cudaMemcpyToSymbol(gq::g_device_status, &z, sizeof(int)));
  }
  int v32 = 0;
  GQ_TRY(gq::tc32::read_status(reset, &v32));
  *status_out = v ? v : v32;
  return GQ_OK;
}

}  // extern "C"
