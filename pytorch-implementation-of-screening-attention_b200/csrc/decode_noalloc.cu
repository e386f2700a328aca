// screen_decode_noalloc: the single-token decode of screen_decode for callers
// that cannot allocate device memory on their serving path -- for example a
// process that must keep its device footprint fixed after start-up (a
// pre-reserved memory budget shared with other tenants), or a plain C /
// foreign-language caller that links only this library and has no device
// allocator of its own to hand us a workspace.
//
// Instead of a caller-provided workspace, the split-K partial sums live in a
// file-scope device array of SCREEN_DECODE_NOALLOC_SCRATCH_BYTES (4 MiB).
// Every GPU that loads the library holds that array until the process exits.
// Host code must not pass the array's name to a kernel (on the host it is only
// a stand-in symbol): the device address is looked up once per device with
// cudaGetSymbolAddress, with that device current, on the first call made on
// that device.  Make that first call before any stream capture.
//
// All calls share the one array, and each call leaves its partials in it.
// Nothing in it needs to start at zero: every split writes all of its
// partial before the finishing kernel reads it.  Calls that overlap on the
// GPU (different streams, or other threads) race on the array and must be
// serialised by the caller.
#include <mutex>
#include "decode.cuh"

namespace {

constexpr size_t kScratchBytes = SCREEN_DECODE_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) float g_decode_scratch[kScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device (nullptr on error).
void* scratch_on_current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || !p) {
      screen::record_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
      return nullptr;
    }
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace

extern "C" {

int screen_decode_noalloc(const screen_decode_args* a, screen_stream_t stream) {
  if (!a) return SCREEN_ERR_INVALID_ARG;
  if (a->dtype != SCREEN_F32 && a->dtype != SCREEN_BF16) return SCREEN_ERR_DTYPE;
  if (a->D != 16 && a->D != 32 && a->D != 64 && a->D != 128) return SCREEN_ERR_HEAD_DIM;
  if (a->B < 0 || a->H < 0 || a->num_splits < 1) return SCREEN_ERR_INVALID_ARG;
  if ((long long)a->B * a->H == 0) return SCREEN_OK;
  if (!a->q || !a->seq_lens || !a->r || !a->w || !a->y || !a->cache.k_pages ||
      !a->cache.v_pages || !a->cache.block_table || a->cache.page_size <= 0 ||
      a->cache.max_blocks <= 0)
    return SCREEN_ERR_INVALID_ARG;
  if (!al16(a->q) || !al16(a->cache.k_pages) || !al16(a->cache.v_pages) || a->q_sb % 4 != 0)
    return SCREEN_ERR_ALIGNMENT;
  // partials: B * H * num_splits * D floats must fit the static array
  const unsigned long long need =
      (unsigned long long)a->B * a->H * a->num_splits * a->D * sizeof(float);
  if (need > kScratchBytes) return SCREEN_ERR_SCRATCH_LIMIT;
  void* scratch = scratch_on_current_device();
  if (!scratch) return SCREEN_ERR_CUDA;
  screen::decode(*a, reinterpret_cast<float*>(scratch), (cudaStream_t)stream);
  return screen::check_launch();
}

}  // extern "C"
