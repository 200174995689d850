// GPTQ sweep for callers that cannot allocate device memory.
//
// gq_gptq_sweep needs scratch space (the working weights in permuted order,
// their codes and one block of errors), and normally the caller provides it.
// Some callers cannot: a host framework may already have reserved almost all
// of the GPU's memory for its own pool (JAX, for instance, preallocates most
// of device memory when it starts), so a cudaMalloc made behind its back
// fails even though the framework could hold the data, and a plain plugin
// interface gives the library no way to borrow from that pool.  cudaFree
// also synchronizes the whole device, which a caller in the middle of
// stream-ordered work may not be allowed to do.
//
// gq_gptq_sweep_static serves those callers from a fixed buffer that lives
// in this file as a __device__ array.  Every GPU that loads the library keeps
// that buffer (kStaticSweepScratchBytes) until the process exits; a sweep
// whose scratch would not fit is rejected with GQ_EINVAL.  The buffer is
// shared by all calls on a device and keeps whatever the last call left in
// it; no part of it has to start at zero, because the sweep writes every
// scratch byte it later reads within the same call.  Two calls whose work
// overlaps on the GPU (different streams, no ordering between them) use the
// same bytes and race -- order such calls, or use gq_gptq_sweep with
// separate workspaces.
//
// Host code must not hand the array's name to a kernel: on the host it is a
// stand-in symbol, not a device address.  The first call on each device (with
// that device current) looks the real address up with cudaGetSymbolAddress
// and caches it together with the CUDA context it was resolved in; make that
// first call before any stream capture begins.  A later call from a different
// context on the same device (after cudaDeviceReset, or from a context the
// caller created) resolves the address again instead of using a stale one.
#include <cuda.h>

#include "gq_common.cuh"

#include <mutex>

namespace gq {

int64_t sweep_ws_bytes(int64_t m, int64_t n);
int sweep_shape_ok(const char* who, int64_t m, int64_t n);

constexpr int64_t kStaticSweepScratchBytes = 32ll * 1024 * 1024;
static_assert(kStaticSweepScratchBytes == GQ_SWEEP_STATIC_SCRATCH_BYTES,
              "header and implementation disagree on the static scratch size");

static __device__ __align__(256) unsigned char g_sweep_scratch[kStaticSweepScratchBytes];

static std::mutex g_scratch_mu;
static void* g_scratch_addr[128] = {};
static CUcontext g_scratch_ctx[128] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// The calling thread's current CUDA context (driver entry point, so the
// library needs no link against libcuda); nullptr when it cannot be read.
static CUcontext current_context() {
  static CtxGetCurrentFn fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(ptr);
    return static_cast<CtxGetCurrentFn>(nullptr);
  }();
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// Device address of g_sweep_scratch on the current device, looked up once per
// (device, context) pair.
static int static_scratch_address(void** out) {
  int dev = -1;
  GQ_CHECK_CUDA(cudaGetDevice(&dev));
  GQ_REQUIRE(dev >= 0 && dev < 128, "gq_gptq_sweep_static: device index %d out of range", dev);
  // nullptr until the runtime has bound a context to this thread; the lookup
  // below binds the device's primary context
  CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr || ctx == nullptr || g_scratch_ctx[dev] != ctx) {
    void* addr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&addr, g_sweep_scratch);
    if (e != cudaSuccess || addr == nullptr)
      return fail(GQ_ECUDA, "gq_gptq_sweep_static: cudaGetSymbolAddress failed on device %d: %s",
                  dev, cudaGetErrorString(e));
    g_scratch_addr[dev] = addr;
    g_scratch_ctx[dev] = current_context();
  }
  *out = g_scratch_addr[dev];
  return GQ_OK;
}

}  // namespace gq

extern "C" int gq_gptq_sweep_static(const float* w, int64_t m, int64_t n, int64_t ldw,
                                    const float* start, const float* u, int64_t ldu,
                                    const int32_t* perm, int w_bits, int group_size, int sym,
                                    int block, const float* group0_scale,
                                    const float* group0_zero, int noprop_cols, float* dequant,
                                    uint8_t* codes, float* scales, float* zeros, int32_t* g_idx,
                                    void* stream) {
  GQ_TRY(gq::sweep_shape_ok("gq_gptq_sweep_static", m, n));  // before any size arithmetic
  const int64_t need = gq::sweep_ws_bytes(m, n);
  GQ_REQUIRE(need <= gq::kStaticSweepScratchBytes,
             "gq_gptq_sweep_static: a %lld x %lld sweep needs %lld bytes of scratch but the "
             "static buffer holds %lld; use gq_gptq_sweep with a caller-provided workspace",
             (long long)m, (long long)n, (long long)need, (long long)gq::kStaticSweepScratchBytes);
  void* scratch = nullptr;
  GQ_TRY(gq::static_scratch_address(&scratch));
  return gq_gptq_sweep(w, m, n, ldw, start, u, ldu, perm, w_bits, group_size, sym, block,
                       group0_scale, group0_zero, noprop_cols, dequant, codes, scales, zeros, g_idx,
                       scratch, gq::kStaticSweepScratchBytes, stream);
}
