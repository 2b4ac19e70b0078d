// An allocation-free entry point: RMSNorm + skinny GEMV with its split-K scratch in a fixed,
// file-scope device array.
//
// Some callers cannot allocate device memory: code running inside a foreign memory pool or a
// host framework that owns every allocation, callers in a restricted context that may not
// call cudaMalloc/cudaFree (and may not pay their synchronisation), or a runtime that must
// start without touching the allocator. pp_norm_gemv_static serves them: the caller passes
// only its inputs and output; the stream-K partial sums and tile counters the kernel needs
// live in g_norm_gemv_scratch below, which every GPU that loads this library holds (about
// 1.2 MB) until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/potpori_b200.h"
#include "pp_common.cuh"
#include "pp_gemv.cuh"

using namespace pp;

namespace {

constexpr int kStaticRows = 8;        // chunk rows (m) the static variant runs
constexpr int kStaticMaxCtas = 148;   // one CTA per SM on a B200
constexpr int kStaticMaxTiles = 8192; // output rows up to 8192 * 128
constexpr size_t kPartialBytes = (size_t)kStaticMaxCtas * 2 * kTileRows * kStaticRows * 4;
constexpr size_t kCounterBytes = (size_t)kStaticMaxTiles * 4;
constexpr size_t kScratchBytes = kPartialBytes + kCounterBytes;

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};  // device address of the array, per device
int g_num_sms[kMaxDevices] = {};
size_t g_smem_budget[kMaxDevices] = {};  // dynamic shared memory the kernel may use, per device

// Messages go where pp_last_error(NULL, ...) reads them.
pp_status static_fail(pp_status st, const char* msg) {
  pp::set_global_error(msg);
  return st;
}

}  // namespace

// The scratch: [kStaticMaxCtas][2][128][8] F32 partial sums, then [kStaticMaxTiles] u32 tile
// counters. In host code this name is only a stand-in for the symbol, not a device address;
// the address comes from cudaGetSymbolAddress at set-up.
static __device__ __align__(256) uint8_t g_norm_gemv_scratch[kScratchBytes];

extern "C" pp_status pp_norm_gemv_static(const uint16_t* w_tiled, const float* x,
                                         const float* norm_w, float eps, uint32_t n, uint32_t k,
                                         uint32_t m, float* y, uint32_t* err, void* stream) {
  if (!w_tiled || !x || !norm_w || !y) return static_fail(PP_E_INVALID, "null argument");
  if (m < 1 || m > (uint32_t)kStaticRows)
    return static_fail(PP_E_INVALID, "m must be 1..8 rows");
  if (k == 0 || k % 8 || n == 0)
    return static_fail(PP_E_INVALID, "k must be a positive multiple of 8 and n positive");
  const uint32_t tiles = (n + kTileRows - 1) / kTileRows;
  if (tiles > (uint32_t)kStaticMaxTiles)
    return static_fail(PP_E_INVALID, "n exceeds the static scratch (8192 tiles of 128 rows)");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return static_fail(PP_E_CUDA, "no current CUDA device");
  using Kern = void (*)(GemvArgs);
  Kern kern = pp_gemv_kernel<kStaticRows, X_RESIDENT_NORM, EPI_STORE>;
  {
    // Once per device, with that device current: the array's device address and the
    // kernel's shared-memory limit. Documented to run before any stream capture.
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_norm_gemv_scratch);
      if (e != cudaSuccess || !p)
        return static_fail(PP_E_CUDA, "cudaGetSymbolAddress failed for the static scratch");
      int optin = 0, sms = 0;
      cudaFuncAttributes fa;
      if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
              cudaSuccess ||
          cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
          cudaFuncGetAttributes(&fa, kern) != cudaSuccess ||
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               optin - (int)fa.sharedSizeBytes) != cudaSuccess)
        return static_fail(PP_E_CUDA, "kernel set-up failed");
      g_num_sms[dev] = sms < kStaticMaxCtas ? sms : kStaticMaxCtas;
      g_smem_budget[dev] = (size_t)optin - fa.sharedSizeBytes;
      g_scratch_ptr[dev] = p;
    }
  }
  uint8_t* scratch = (uint8_t*)g_scratch_ptr[dev];
  cudaStream_t st = (cudaStream_t)stream;

  GemvArgs a = {};
  a.w = w_tiled;
  a.n_out = (int32_t)n;
  a.n_packed = (int32_t)(tiles * kTileRows);
  a.k = (int32_t)k;
  a.kchunks = (int32_t)((k + kChunkK - 1) / kChunkK);
  a.kp = a.kchunks * kChunkK;
  a.tiles = (int32_t)tiles;
  a.x = x;
  a.ldx = (int32_t)k;
  a.norm_w = norm_w;
  a.eps = eps;
  a.out = y;
  a.ldo = (int32_t)n;
  a.partials = (float*)scratch;
  a.tile_cnt = (uint32_t*)(scratch + kPartialBytes);
  a.m_rows = (int32_t)m;
  // Non-finite x values and an expired bounded wait (ST_NONFINITE_IN, ST_TIMEOUT) are ORed
  // into the caller's error word.
  a.check_input = 1;
  a.status = (int32_t*)err;

  using Lay = GemvSmem<kStaticRows, X_RESIDENT_NORM>;
  const size_t budget = g_smem_budget[dev];
  int ns = 12;
  while (ns > 2 && Lay::total(ns, a.kp) > budget) --ns;
  if (Lay::total(ns, a.kp) > budget)
    return static_fail(PP_E_INVALID, "k too large for the kernel's shared memory");
  a.nstages = ns;

  // Tile counters must start at zero; a memset allocates nothing.
  if (cudaMemsetAsync(a.tile_cnt, 0, (size_t)tiles * 4, st) != cudaSuccess)
    return static_fail(PP_E_CUDA, "clearing the tile counters failed");
  const int64_t T = (int64_t)tiles * a.kchunks;
  const int grid = (int)(T < g_num_sms[dev] ? T : g_num_sms[dev]);
  kern<<<grid, kGemvThreads, Lay::total(ns, a.kp), st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_fail(PP_E_CUDA, cudaGetErrorString(e));
  return PP_OK;
}
