// Library-wide plumbing: error strings, version, device properties.
#include "gq_common.cuh"

#include <atomic>
#include <cstring>

namespace gq {

static thread_local char g_last_error[1024] = "";
static std::atomic<long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

const char* last_error() { return g_last_error; }

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// Grid cap for the persistent tensor-core kernels launched by this host thread.
static thread_local int g_cta_budget = 0;

int cta_budget() {
  const int n = sm_count();
  return (g_cta_budget > 0 && g_cta_budget < n) ? g_cta_budget : n;
}

// Statistics kernels on CTA pairs (1) or one CTA per tile (0), this host thread.
static thread_local int g_pair_kernels = 1;

bool pair_kernels() { return g_pair_kernels != 0; }

// Copy the upper triangle (j > i) of h into the lower triangle.  Tiled
// through shared memory so both the read and the write are coalesced.
__global__ void symmetrize_upper_kernel(float* __restrict__ h, int64_t d, int64_t ldh) {
  __shared__ float tile[32][33];
  int64_t bi = blockIdx.y, bj = blockIdx.x;  // output tile (bi, bj) in the lower triangle
  if (bj > bi) return;
  int tx = threadIdx.x, ty = threadIdx.y;    // 32 x 8
  // source: tile (bj, bi) of the upper triangle
  for (int r = ty; r < 32; r += 8) {
    int64_t i = bj * 32 + r, j = bi * 32 + tx;
    tile[r][tx] = (i < d && j < d) ? h[i * ldh + j] : 0.f;
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    int64_t i = bi * 32 + r, j = bj * 32 + tx;  // destination (i, j), i > j
    if (i < d && j < d && i > j) h[i * ldh + j] = tile[tx][r];
  }
}

// dst[c][r] = src[r][c] for a rows x cols block (tiled through shared memory).
__global__ void transpose2d_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
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

int transpose2d(const float* src, int64_t rows, int64_t cols, int64_t lds, float* dst, int64_t ldd,
                cudaStream_t st) {
  if (rows == 0 || cols == 0) return GQ_OK;
  dim3 grid((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32));
  transpose2d_kernel<<<grid, dim3(32, 8), 0, st>>>(src, rows, cols, lds, dst, ldd);
  return check_launch("transpose2d");
}

int symmetrize_upper(float* h, int64_t d, int64_t ldh, cudaStream_t st) {
  if (d <= 1) return GQ_OK;
  int64_t nt = ceil_div(d, 32);
  dim3 grid((unsigned)nt, (unsigned)nt);
  symmetrize_upper_kernel<<<grid, dim3(32, 8), 0, st>>>(h, d, ldh);
  return check_launch("symmetrize_upper");
}

}  // namespace gq

extern "C" {

int gq_version(void) { return 100; }

const char* gq_last_error(void) { return gq::last_error(); }

long long gq_launch_count(void) { return gq::g_launches.load(std::memory_order_relaxed); }

int gq_symmetrize_upper(float* h, int64_t d, int64_t ldh, void* stream) {
  GQ_REQUIRE(h != nullptr && d >= 0 && ldh >= d, "gq_symmetrize_upper: bad arguments (d=%lld ldh=%lld)",
             (long long)d, (long long)ldh);
  return gq::symmetrize_upper(h, d, ldh, gq::as_stream(stream));
}

}  // extern "C"

extern "C" int gq_set_cta_budget(int n) {
  GQ_REQUIRE(n >= 0, "gq_set_cta_budget: negative budget");
  gq::g_cta_budget = n;
  return GQ_OK;
}

extern "C" int gq_set_pair_kernels(int enable) {
  GQ_REQUIRE(enable == 0 || enable == 1, "gq_set_pair_kernels: enable must be 0 or 1");
  gq::g_pair_kernels = enable;
  return GQ_OK;
}
