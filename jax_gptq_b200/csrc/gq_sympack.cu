// Packed upper triangle of a symmetric d x d float32 matrix, for summing
// token-sharded Hessians across GPUs with half the bytes of the full matrix
// (H = sum_r X_r^T X_r, stats.py:16-17, is symmetric on every rank).
//
// Layout: 128-row blocks b = 0, 1, ...; block b holds rows [128 b, 128 b +
// rows_b) from column 128 b to d - 1, row-major, one after another.  Every
// block but the last has 128 rows, so block b starts at
//   off_b = 128 (b d - 128 b (b - 1) / 2)
// and the whole buffer has off_{nb-1} + rows_last (d - 128 (nb - 1)) floats,
// about d^2 / 2 + 64 d.  The diagonal 128 x 128 tiles are stored whole (both
// triangles), which keeps every packed row one contiguous run.
//
// Unpacking takes only the entries on or above the diagonal and mirrors them,
// so the result is exactly symmetric even where a reduction summed the two
// copies of an entry inside a diagonal tile in different orders.
#include "gq_common.cuh"

namespace gq {

constexpr int64_t SP_ROWS = 128;

__host__ __device__ inline int64_t sym_block_offset(int64_t d, int64_t b) {
  return SP_ROWS * (b * d - SP_ROWS * b * (b - 1) / 2);
}

int64_t sym_packed_size(int64_t d) {
  if (d <= 0) return 0;
  const int64_t nb = ceil_div(d, SP_ROWS);
  const int64_t last = nb - 1;
  const int64_t rows_last = d - SP_ROWS * last;
  return sym_block_offset(d, last) + rows_last * (d - SP_ROWS * last);
}

// one CTA per row r: packed row = h[r][128 b : d]
__global__ void sym_pack_kernel(const float* __restrict__ h, int64_t d, int64_t ldh,
                                float* __restrict__ packed) {
  const int64_t r = blockIdx.x;
  const int64_t b = r / SP_ROWS, c0 = SP_ROWS * b;
  const int64_t width = d - c0;
  const float* src = h + r * ldh + c0;
  float* dst = packed + sym_block_offset(d, b) + (r - c0) * width;
  for (int64_t c = threadIdx.x; c < width; c += blockDim.x) dst[c] = src[c];
}

// one CTA per row r: h[r][c] for c >= r from the packed row (the mirror to
// the lower triangle follows)
__global__ void sym_unpack_kernel(const float* __restrict__ packed, int64_t d,
                                  float* __restrict__ h, int64_t ldh) {
  const int64_t r = blockIdx.x;
  const int64_t b = r / SP_ROWS, c0 = SP_ROWS * b;
  const int64_t width = d - c0;
  const float* src = packed + sym_block_offset(d, b) + (r - c0) * width;
  float* dst = h + r * ldh + c0;
  for (int64_t c = (r - c0) + threadIdx.x; c < width; c += blockDim.x) dst[c] = src[c];
}

int symmetrize_upper(float* h, int64_t d, int64_t ldh, cudaStream_t st);

int sym_pack(const float* h, int64_t d, int64_t ldh, float* packed, cudaStream_t st) {
  if (d == 0) return GQ_OK;
  sym_pack_kernel<<<(unsigned)d, 256, 0, st>>>(h, d, ldh, packed);
  return check_launch("sym_pack");
}

int sym_unpack(const float* packed, int64_t d, float* h, int64_t ldh, cudaStream_t st) {
  if (d == 0) return GQ_OK;
  sym_unpack_kernel<<<(unsigned)d, 256, 0, st>>>(packed, d, h, ldh);
  GQ_TRY(check_launch("sym_unpack"));
  return symmetrize_upper(h, d, ldh, st);
}

}  // namespace gq

extern "C" {

int64_t gq_sym_packed_size(int64_t d) { return gq::sym_packed_size(d); }

int gq_sym_pack_upper(const float* h, int64_t d, int64_t ldh, float* packed, void* stream) {
  GQ_REQUIRE(d >= 0 && d <= (int64_t)INT32_MAX, "gq_sym_pack_upper: bad d %lld", (long long)d);
  GQ_REQUIRE(d == 0 || (h != nullptr && packed != nullptr && ldh >= d),
             "gq_sym_pack_upper: bad arguments (d=%lld ldh=%lld)", (long long)d, (long long)ldh);
  return gq::sym_pack(h, d, ldh, packed, gq::as_stream(stream));
}

int gq_sym_unpack_upper(const float* packed, int64_t d, float* h, int64_t ldh, void* stream) {
  GQ_REQUIRE(d >= 0 && d <= (int64_t)INT32_MAX, "gq_sym_unpack_upper: bad d %lld", (long long)d);
  GQ_REQUIRE(d == 0 || (h != nullptr && packed != nullptr && ldh >= d),
             "gq_sym_unpack_upper: bad arguments (d=%lld ldh=%lld)", (long long)d, (long long)ldh);
  return gq::sym_unpack(packed, d, h, ldh, gq::as_stream(stream));
}

}  // extern "C"
