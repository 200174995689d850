// Packed quantized-weight format.  The reference returns only dequantized
// floats (quant.py:37); this stores what a quantized checkpoint needs:
//   packed [m, ldp] uint32: row r's codes in original column order as one
//     little-endian bit stream, code c in bits [c*bits, (c+1)*bits), word w
//     holding stream bits [32w, 32w + 32); words = ceil(n * bits / 32);
//   scales, zeros [m, n_groups] float32 and g_idx [n] int32 as the sweep
//     returns them (groups in permuted order, g_idx[c] = group of column c).
// Dequantization reproduces the sweep's float32 arithmetic exactly:
// (code + qmin - zero) * scale with explicit round-to-nearest operations.
#include "gq_common.cuh"
#include "gq_quant.cuh"

namespace gq {

__global__ void pack_codes_kernel(const uint8_t* __restrict__ codes, int64_t m, int64_t n,
                                  int64_t ldc, int bits, uint32_t* __restrict__ packed,
                                  int64_t ldp, int64_t words) {
  const uint32_t mask = (1u << bits) - 1u;
  for (int64_t r = blockIdx.y; r < m; r += gridDim.y)
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < words;
       w += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t* row = codes + r * ldc;
    const int64_t base = 32 * w;
    const int64_t j0 = base / bits;
    const int64_t j1 = min(n - 1, (base + 31) / bits);
    uint64_t v = 0;
    for (int64_t j = j0; j <= j1; ++j) {
      const uint64_t code = row[j] & mask;
      const int64_t pos = j * bits - base;
      v |= (pos >= 0) ? (code << pos) : (code >> (-pos));
    }
    packed[r * ldp + w] = (uint32_t)v;
  }
}

__global__ void unpack_dequant_kernel(const uint32_t* __restrict__ packed, int64_t m, int64_t n,
                                      int64_t ldp, int bits, float qmin,
                                      const float* __restrict__ scales,
                                      const float* __restrict__ zeros, int64_t n_groups,
                                      const int32_t* __restrict__ g_idx,
                                      float* __restrict__ dequant, uint8_t* __restrict__ codes) {
  const uint32_t mask = (1u << bits) - 1u;
  for (int64_t r = blockIdx.y; r < m; r += gridDim.y)
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < n;
       c += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t* row = packed + r * ldp;
    const int64_t bit = c * bits;
    const int64_t w = bit >> 5;
    const int off = (int)(bit & 31);
    uint64_t v = row[w];
    if (off + bits > 32) v |= (uint64_t)row[w + 1] << 32;
    const uint32_t code = (uint32_t)(v >> off) & mask;
    if (codes) codes[r * n + c] = (uint8_t)code;
    if (dequant) {
      const int64_t gi = g_idx[c];
      const float s = scales[r * n_groups + gi], z = zeros[r * n_groups + gi];
      const float q = __fadd_rn((float)code, qmin);
      dequant[r * n + c] = __fmul_rn(__fsub_rn(q, z), s);
    }
  }
}

}  // namespace gq

extern "C" {

int64_t gq_packed_words(int64_t n, int bits) {
  if (n < 0 || bits < 1 || bits > 8) return -1;
  return (n * bits + 31) / 32;
}

int gq_pack_codes(const uint8_t* codes, int64_t m, int64_t n, int64_t ldc, int bits,
                  uint32_t* packed, int64_t ldp, void* stream) {
  GQ_REQUIRE(bits >= 1 && bits <= 8, "gq_pack_codes: bits must be 1..8");
  GQ_REQUIRE(m >= 0 && n >= 0 && ldc >= n, "gq_pack_codes: bad shape");
  const int64_t words = gq_packed_words(n, bits);
  GQ_REQUIRE(ldp >= words, "gq_pack_codes: ldp < %lld words", (long long)words);
  if (m == 0 || n == 0) return GQ_OK;
  GQ_REQUIRE(codes != nullptr && packed != nullptr, "gq_pack_codes: NULL buffer");
  dim3 grid((unsigned)std::min<int64_t>(gq::ceil_div(words, 256), 64),
            (unsigned)std::min<int64_t>(m, 65535));
  gq::pack_codes_kernel<<<grid, 256, 0, gq::as_stream(stream)>>>(codes, m, n, ldc, bits, packed,
                                                                 ldp, words);
  return gq::check_launch("gq_pack_codes");
}

int gq_unpack_dequant(const uint32_t* packed, int64_t m, int64_t n, int64_t ldp, int bits, int sym,
                      const float* scales, const float* zeros, int64_t n_groups,
                      const int32_t* g_idx, float* dequant, uint8_t* codes, void* stream) {
  GQ_REQUIRE(bits >= 1 && bits <= 8 && (!sym || bits >= 2), "gq_unpack_dequant: bad bits");
  GQ_REQUIRE(m >= 0 && n >= 0 && ldp >= gq_packed_words(n, bits), "gq_unpack_dequant: bad shape");
  GQ_REQUIRE(dequant == nullptr || (scales && zeros && g_idx && n_groups > 0),
             "gq_unpack_dequant: dequant needs scales, zeros and g_idx");
  if (m == 0 || n == 0) return GQ_OK;
  GQ_REQUIRE(packed != nullptr, "gq_unpack_dequant: NULL packed");
  const gq::QParams qp = gq::make_qparams(bits, sym);
  dim3 grid((unsigned)std::min<int64_t>(gq::ceil_div(n, 256), 64),
            (unsigned)std::min<int64_t>(m, 65535));
  gq::unpack_dequant_kernel<<<grid, 256, 0, gq::as_stream(stream)>>>(
      packed, m, n, ldp, bits, qp.qmin, scales, zeros, n_groups, g_idx, dequant, codes);
  return gq::check_launch("gq_unpack_dequant");
}

}  // extern "C"
