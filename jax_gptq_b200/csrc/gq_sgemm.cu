// FP32 GEMM on the CUDA cores (C = alpha op(A) op(B) + beta C, row-major).
// 128x128 output tile per CTA, K step 8, 256 threads with an 8x8 register
// micro-tile each, double-buffered shared memory.  Used where float32
// accuracy is required (GPTQ lazy trailing update, Cholesky / triangular
// inverse updates, QR compact-WY updates, fp32 activation statistics).
#include "gq_common.cuh"

namespace gq {

constexpr int SG_BM = 128, SG_BN = 128, SG_BK = 8, SG_THREADS = 256;

template <bool TA, bool TB>
__global__ void __launch_bounds__(SG_THREADS)
sgemm_kernel(int64_t M, int64_t N, int64_t K, float alpha, const float* __restrict__ A, int64_t lda,
             const float* __restrict__ B, int64_t ldb, float beta, float* __restrict__ C,
             int64_t ldc, int uplo) {
  const int64_t bm = blockIdx.y, bn = blockIdx.x;
  const int64_t row0 = bm * SG_BM, col0 = bn * SG_BN;
  if (uplo == 1 && col0 > row0 + SG_BM - 1) return;
  if (uplo == 2 && col0 + SG_BN - 1 < row0) return;

  __shared__ __align__(16) float As[2][SG_BK][SG_BM];
  __shared__ __align__(16) float Bs[2][SG_BK][SG_BN];

  const int tid = threadIdx.x;
  // Load mapping: each thread brings 4 elements of the A tile and 4 of B.
  // A tile element (mm, kk): for !TA read along k (kk fastest), for TA along m.
  float ra[4], rb[4];

  auto load_a = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int e = tid + i * SG_THREADS;  // 0..1023
      int mm, kk;
      if (!TA) { mm = e >> 3; kk = e & 7; } else { kk = e >> 7; mm = e & 127; }
      int64_t gm = row0 + mm, gk = k0 + kk;
      float v = 0.f;
      if (gm < M && gk < K) v = TA ? A[gk * lda + gm] : A[gm * lda + gk];
      ra[i] = v;
    }
  };
  auto store_a = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int e = tid + i * SG_THREADS;
      int mm, kk;
      if (!TA) { mm = e >> 3; kk = e & 7; } else { kk = e >> 7; mm = e & 127; }
      As[buf][kk][mm] = ra[i];
    }
  };
  auto load_b = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int e = tid + i * SG_THREADS;
      int nn, kk;
      if (!TB) { kk = e >> 7; nn = e & 127; } else { nn = e >> 3; kk = e & 7; }
      int64_t gn = col0 + nn, gk = k0 + kk;
      float v = 0.f;
      if (gn < N && gk < K) v = TB ? B[gn * ldb + gk] : B[gk * ldb + gn];
      rb[i] = v;
    }
  };
  auto store_b = [&](int buf) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int e = tid + i * SG_THREADS;
      int nn, kk;
      if (!TB) { kk = e >> 7; nn = e & 127; } else { nn = e >> 3; kk = e & 7; }
      Bs[buf][kk][nn] = rb[i];
    }
  };

  // Compute mapping: 16 x 16 threads, each owns rows {ty*4 + i, 64 + ty*4 + i}
  // and cols {tx*4 + j, 64 + tx*4 + j} (two float4 groups -> conflict-free LDS.128).
  const int tx = tid & 15, ty = tid >> 4;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int64_t nk = ceil_div(K, SG_BK);
  load_a(0);
  load_b(0);
  store_a(0);
  store_b(0);
  __syncthreads();

  for (int64_t kt = 0; kt < nk; ++kt) {
    const int buf = (int)(kt & 1);
    if (kt + 1 < nk) {
      load_a((kt + 1) * SG_BK);
      load_b((kt + 1) * SG_BK);
    }
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kt + 1 < nk) {
      store_a(buf ^ 1);
      store_b(buf ^ 1);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int64_t gm = row0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int64_t gn = col0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn >= N) continue;
      float* cp = C + gm * ldc + gn;
      float v = alpha * acc[i][j];
      if (beta != 0.f) v = fmaf(beta, *cp, v);
      *cp = v;
    }
  }
}

namespace tc32 {
bool eligible(int ta, int tb, int64_t M, int64_t N, int64_t K, const float* A, int64_t lda,
              const float* B, int64_t ldb, const float* C, int64_t ldc);
int launch(int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
           const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int uplo, int tri,
           cudaStream_t st);
}  // namespace tc32

int sgemm_simt(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A,
               int64_t lda, const float* B, int64_t ldb, float beta, float* C, int64_t ldc,
               int uplo, cudaStream_t st);

// fp32 GEMM used throughout the library: the tcgen05 3xTF32 kernel when the
// shape and alignment allow it, the CUDA-core kernel otherwise.
int sgemm(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A, int64_t lda,
          const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int uplo, cudaStream_t st) {
  if (M == 0 || N == 0) return GQ_OK;
  if (tc32::eligible(ta, tb, M, N, K, A, lda, B, ldb, C, ldc))
    return tc32::launch(tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, uplo, 0, st);
  return sgemm_simt(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, uplo, st);
}

// sgemm with a triangular operand whose zero triangle is stored as zeros and
// starts on 128 boundaries (tri: 1 A upper, 2 A lower, 3 B lower, 4 B upper;
// "upper" = zero below the diagonal, B given [N, K]): the
// tensor-core path skips the all-zero k-slices of each tile; the result is the
// same as the full product.
int sgemm_tri(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A,
              int64_t lda, const float* B, int64_t ldb, float beta, float* C, int64_t ldc, int tri,
              cudaStream_t st) {
  if (M == 0 || N == 0) return GQ_OK;
  if (tc32::eligible(ta, tb, M, N, K, A, lda, B, ldb, C, ldc))
    return tc32::launch(tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, 0, tri, st);
  return sgemm_simt(ta, tb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, 0, st);
}

int sgemm_simt(int ta, int tb, int64_t M, int64_t N, int64_t K, float alpha, const float* A,
               int64_t lda, const float* B, int64_t ldb, float beta, float* C, int64_t ldc,
               int uplo, cudaStream_t st) {
  if (M == 0 || N == 0) return GQ_OK;
  dim3 grid((unsigned)ceil_div(N, SG_BN), (unsigned)ceil_div(M, SG_BM));
  if (grid.y > 65535) return fail(GQ_EUNSUPPORTED, "gq_sgemm: M=%lld too large", (long long)M);
  if (ta == 0 && tb == 0)
    sgemm_kernel<false, false><<<grid, SG_THREADS, 0, st>>>(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  else if (ta == 0 && tb == 1)
    sgemm_kernel<false, true><<<grid, SG_THREADS, 0, st>>>(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  else if (ta == 1 && tb == 0)
    sgemm_kernel<true, false><<<grid, SG_THREADS, 0, st>>>(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  else
    sgemm_kernel<true, true><<<grid, SG_THREADS, 0, st>>>(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  return check_launch("gq_sgemm");
}

}  // namespace gq

extern "C" {

int gq_sgemm(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, float alpha,
             const float* a, int64_t lda, const float* b, int64_t ldb, float beta, float* c,
             int64_t ldc, int uplo, void* stream) {
  GQ_REQUIRE(M >= 0 && N >= 0 && K >= 0, "gq_sgemm: negative size");
  GQ_REQUIRE(uplo >= 0 && uplo <= 2, "gq_sgemm: uplo must be 0, 1 or 2");
  GQ_REQUIRE(ldc >= N, "gq_sgemm: ldc < N");
  GQ_REQUIRE(lda >= (trans_a ? M : K), "gq_sgemm: lda too small");
  GQ_REQUIRE(ldb >= (trans_b ? K : N), "gq_sgemm: ldb too small");
  return gq::sgemm(trans_a ? 1 : 0, trans_b ? 1 : 0, M, N, K, alpha, a, lda, b, ldb, beta, c, ldc,
                   uplo, gq::as_stream(stream));
}

int gq_sgemm_simt(int trans_a, int trans_b, int64_t M, int64_t N, int64_t K, float alpha,
                  const float* a, int64_t lda, const float* b, int64_t ldb, float beta, float* c,
                  int64_t ldc, int uplo, void* stream) {
  GQ_REQUIRE(M >= 0 && N >= 0 && K >= 0, "gq_sgemm_simt: negative size");
  GQ_REQUIRE(uplo >= 0 && uplo <= 2, "gq_sgemm_simt: uplo must be 0, 1 or 2");
  GQ_REQUIRE(ldc >= N && lda >= (trans_a ? M : K) && ldb >= (trans_b ? K : N),
             "gq_sgemm_simt: leading dimension too small");
  return gq::sgemm_simt(trans_a ? 1 : 0, trans_b ? 1 : 0, M, N, K, alpha, a, lda, b, ldb, beta, c,
                        ldc, uplo, gq::as_stream(stream));
}

int gq_syrk_f32(const float* x, int64_t tokens, int64_t d, int64_t ldx, float* h, int64_t ldh,
                int accumulate, void* stream) {
  GQ_REQUIRE(tokens >= 0 && d >= 0 && ldx >= d && ldh >= d, "gq_syrk_f32: bad shape");
  cudaStream_t st = gq::as_stream(stream);
  GQ_TRY(gq::sgemm(1, 0, d, d, tokens, 1.f, x, ldx, x, ldx, accumulate ? 1.f : 0.f, h, ldh, 2, st));
  return gq_symmetrize_upper(h, d, ldh, stream);
}

int gq_gemm_tn_f32(const float* xa, int64_t lda, const float* xb, int64_t ldb, int64_t tokens,
                   int64_t da, int64_t db, float* g, int64_t ldg, int accumulate, void* stream) {
  GQ_REQUIRE(tokens >= 0 && da >= 0 && db >= 0 && lda >= da && ldb >= db && ldg >= db,
             "gq_gemm_tn_f32: bad shape");
  return gq::sgemm(1, 0, da, db, tokens, 1.f, xa, lda, xb, ldb, accumulate ? 1.f : 0.f, g, ldg, 0,
                   gq::as_stream(stream));
}

}  // extern "C"
