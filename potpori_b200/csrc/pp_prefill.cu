// Prompt-sized projection on the 5th-generation tensor cores (tcgen05 + TMEM):
//   y[t][j] = sum_c W[j][c] * x[t][c]   for t < T rows (a prompt chunk), j < n, c < k,
// W BF16 in the shards' tiled layout, x and y F32 — the linear of src/qwen/model.rs:166-183
// at the M = 2048 prefill of the 8-stage workload, where the shape is a dense contraction.
//
// Layout and arithmetic. A tiled weight block (128 rows x 64 columns, the 16-byte unit u of
// row r at u ^ (r & 7)) is already the canonical K-major SWIZZLE_128B operand of the MMA
// (8-row atoms of 1024 bytes), so one 1-D bulk copy moves it into shared memory unchanged.
// The activations are split x = hi + lo (hi = bf16(x), lo = bf16(x - hi), about 2^-17
// relative) by pp_rows_split_kernel into blocks of the same form (128 rows x 64 columns per
// part), and every K step issues two MMAs, W.hi and W.lo, into one F32 accumulator: the
// products of BF16 are exact and the sum is the reference's F32 arithmetic to its rounding.
//
// Kernel (persistent, one CTA per SM looping over 128 weight rows x 128 activation rows units,
// 192 threads):
//  * warp 0, one thread: per 64-column chunk of every unit of the CTA, the weight block
//    (16 KB) and the two activation parts (16 KB each) into a ring of four 48 KB stages (bulk
//    copies, mbarrier transaction counts; no multicast), without draining between units;
//  * warp 1: allocates 256 TMEM columns (two 128 x 128 F32 accumulators), and one thread
//    issues tcgen05.mma (kind::f16, M = 128, N = 128, K = 16) into the accumulator of the
//    unit, returns each stage to the producer with tcgen05.commit on its empty barrier and
//    marks the accumulator full when the unit's last chunk is in;
//  * warps 2-5: tcgen05.ld a full accumulator (warp w reads TMEM lanes 32 (w % 4) .. + 31),
//    store y with consecutive lanes on consecutive j, and hand the accumulator back, so one
//    unit's epilogue runs under the next unit's MMAs.
// Every wait is bounded; a wait that expires sets the error word and the CTA still frees
// its TMEM and lets its copies land before it exits.
#include <cuda_runtime.h>

#include <cstdio>

#include "../../include/potpori_b200.h"
#include "pp_common.cuh"
#include "pp_rows_blocks.cuh"

using namespace pp;

namespace pp {

constexpr int kRgM = 128;                      // weight rows per tile (TMEM lanes)
constexpr int kRgWBytes = kRgM * kChunkK * 2;  // 16 KB weight block
constexpr int kRgStage = kRgWBytes + 2 * kRgXBytes;
constexpr int kRgStages = 4;  // 4 x 48 KB: a refill from L2 outlasts one stage's MMAs
constexpr int kRgThreads = 192;
constexpr size_t kRgSmem = (size_t)kRgStages * kRgStage + 256 + 1024;

// Instruction descriptor of tcgen05.mma kind::f16: F32 accumulator, BF16 A and B, both
// K-major, N = 128 (bits 17-22: N / 8), M = 128 (bits 24-28: M / 16).
constexpr uint32_t kRgIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kRgN >> 3) << 17) |
                              ((uint32_t)(kRgM >> 4) << 24);

// Shared-memory matrix descriptor of a K-major SWIZZLE_128B operand at byte address saddr
// (1024-aligned): start >> 4, leading offset 1 (unused for this swizzle), stride between
// 8-row atoms 1024 B (>> 4 = 64), descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t rg_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)64 << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void rg_mma(uint32_t tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
      "l"(adesc), "l"(bdesc), "r"(kRgIdesc), "r"(acc));
}
__device__ __forceinline__ void rg_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void rg_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void rg_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Splits F32 rows x[t][c] (row stride ldx) into the MMA's activation blocks (the layout of
// pp_rows_blocks.cuh); rows past T and columns past k are zero. One thread per (row, unit).
__global__ void pp_rows_split_kernel(const float* x, int32_t ldx, int32_t T, int32_t k,
                                     int32_t kchunks, int32_t tblocks, uint8_t* xs) {
  const int64_t units = (int64_t)tblocks * kRgN * kchunks * 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < units;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / (kchunks * 8);
    const int u = (int)(i - row * (kchunks * 8));  // unit over the whole padded row
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int col = u * 8 + e;
      v[e] = (row < T && col < k) ? x[row * (int64_t)ldx + col] : 0.f;
    }
    rows_store_unit(xs, kchunks, (int)row, u, v);
  }
}

// Persistent: one CTA per SM (gridDim.x <= units), kRgThreads threads, kRgSmem bytes of
// dynamic shared memory. Work unit u = (weight tile u / tblocks, token block u % tblocks): token
// blocks vary fastest, so the CTAs in flight share weight tiles (each read from DRAM about
// once) and the activations stay in L2. CTA b takes u = b, b + gridDim.x, ...; its producer
// streams the chunks of all its units through the stage ring without draining between them,
// and two TMEM accumulators let the epilogue of one unit run under the MMAs of the next.
__global__ void __launch_bounds__(kRgThreads, 1)
    pp_rows_gemm_kernel(const uint16_t* w, const uint8_t* xs, float* y, int32_t ldy, int32_t n,
                        int32_t T, int32_t kchunks, int32_t tblocks, int32_t units, int32_t accumulate,
                        uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + (size_t)kRgStages * kRgStage);
  uint64_t* empty = full + kRgStages;
  uint64_t* afull = empty + kRgStages;  // [2] accumulator b holds a finished unit
  uint64_t* aempty = afull + 2;         // [2] accumulator b was drained by the epilogue
  uint64_t* done = aempty + 2;          // every MMA of this CTA has completed
  uint32_t* tmem_slot = (uint32_t*)(done + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kRgStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&afull[b], 1);
      mbar_init(&aempty[b], 4);  // the four epilogue warps
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {  // the whole warp allocates; the address lands in shared memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(2 * kRgN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  rg_fence_before();
  __syncthreads();
  rg_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;  // chunks issued by this CTA
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int tb = u % tblocks, tile = u / tblocks;
        for (int c = 0; c < kchunks; ++c) {
          const int s = it % kRgStages;
          const uint32_t use = (uint32_t)(it / kRgStages);
          if (it >= kRgStages && !mbar_wait(&empty[s], (use - 1) & 1u)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + (size_t)s * kRgStage;
          mbar_arrive_expect_tx(&full[s], kRgStage);
          bulk_load(st, w + ((size_t)tile * kchunks + c) * (kRgM * kChunkK), kRgWBytes, &full[s]);
          const uint8_t* xb = xs + ((size_t)tb * kchunks + c) * 2 * kRgXBytes;
          bulk_load(st + kRgWBytes, xb, kRgXBytes, &full[s]);
          bulk_load(st + kRgWBytes + kRgXBytes, xb + kRgXBytes, kRgXBytes, &full[s]);
          ++it;
        }
      }
      if (!ok) {
        atomicOr(err, 1u);
        for (int c = it > kRgStages ? it - kRgStages : 0; c < it; ++c)
          mbar_wait(&full[c % kRgStages], (uint32_t)(c / kRgStages) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      int it = 0, i = 0;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++i) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait(&aempty[b], (uint32_t)((i >> 1) - 1) & 1u)) {
          ok = false;
          break;
        }
        rg_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * kRgN);
        for (int c = 0; c < kchunks; ++c, ++it) {
          const int s = it % kRgStages;
          if (!mbar_wait(&full[s], (uint32_t)(it / kRgStages) & 1u)) {
            ok = false;
            break;
          }
          rg_fence_after();
          const uint32_t base = smem_u32(smem + (size_t)s * kRgStage);
          const uint64_t a = rg_desc(base), bh = rg_desc(base + kRgWBytes),
                         bl = rg_desc(base + kRgWBytes + kRgXBytes);
#pragma unroll
          for (int j = 0; j < kChunkK / 16; ++j) {  // K = 16 per MMA: +32 bytes = +2 in the descriptor
            rg_mma(acc, a + 2 * j, bh + 2 * j, (c | j) != 0);
            rg_mma(acc, a + 2 * j, bl + 2 * j, 1u);
          }
          rg_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (ok) rg_commit(&afull[b]);  // the unit's accumulator is complete
      }
      if (!ok) atomicOr(err, 2u);
      rg_commit(done);
      mbar_wait(done, 0);  // no MMA of this CTA still runs when TMEM is freed
    }
  } else {
    // Epilogue: warp w reads TMEM lanes 32 (w % 4) ..; lane = weight row, column = row of x.
    const int q = warp & 3;
    int i = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++i) {
      const int b = i & 1, tb = u % tblocks, tile = u / tblocks;
      if (!mbar_wait(&afull[b], (uint32_t)(i >> 1) & 1u)) {
        if (lane == 0) atomicOr(err, 4u);
        break;
      }
      rg_fence_after();
      const int j = tile * kRgM + q * 32 + lane;
      for (int cc = 0; cc < kRgN / 32; ++cc) {
        uint32_t v[32];
        const uint32_t addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * kRgN + cc * 32);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, "
            "%10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, "
            "%26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
              "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]),
              "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]),
              "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
              "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
              "=r"(v[30]), "=r"(v[31])
            : "r"(addr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (j < n) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int t = tb * kRgN + cc * 32 + e;
            if (t < T && accumulate)  // every load in flight before the first store
              v[e] = __float_as_uint(y[(size_t)t * ldy + j] + __uint_as_float(v[e]));
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int t = tb * kRgN + cc * 32 + e;
            if (t < T) y[(size_t)t * ldy + j] = __uint_as_float(v[e]);
          }
        }
      }
      rg_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&aempty[b]);  // the MMA thread may refill accumulator b
    }
  }
  rg_fence_before();
  __syncthreads();
  if (warp == 1) {
    rg_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(2 * kRgN));
  }
}

}  // namespace pp

namespace {
pp_status rg_fail(pp_status st, const char* msg) {
  pp::set_global_error(msg);
  return st;
}
}  // namespace

extern "C" uint64_t pp_rows_gemm_work_bytes(uint32_t t, uint32_t k) {
  const uint64_t tblocks = (t + kRgN - 1) / kRgN, kchunks = (k + kChunkK - 1) / kChunkK;
  return tblocks * kchunks * 2 * (uint64_t)kRgXBytes;
}

namespace pp {
pp_status rows_gemm_blocks(const uint16_t* w_tiled, uint32_t n, uint32_t k, const uint8_t* xs,
                           uint32_t t, float* y, uint32_t ldy, bool accumulate, uint32_t* err,
                           cudaStream_t st) {
  if (!w_tiled || !xs || !y || !err) return rg_fail(PP_E_INVALID, "null argument");
  if (n == 0 || k == 0 || t == 0 || n > (1u << 24) || k > (1u << 20) || t > (1u << 20) || ldy < n)
    return rg_fail(PP_E_INVALID, "sizes out of range");
  if ((uintptr_t)w_tiled % 16 || (uintptr_t)xs % 1024)
    return rg_fail(PP_E_INVALID, "w_tiled must be 16-byte and work 1024-byte aligned");
  static bool attr_done[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return rg_fail(PP_E_CUDA, "no current device");
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(pp_rows_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kRgSmem) != cudaSuccess)
      return rg_fail(PP_E_CUDA, "cannot reserve the GEMM's shared memory");
    attr_done[dev] = true;
  }
  const int kchunks = (int)((k + kChunkK - 1) / kChunkK);
  const int tblocks = (int)((t + kRgN - 1) / kRgN);
  const int tiles = (int)((n + kRgM - 1) / kRgM);
  const int units = tiles * tblocks;
  static int num_sms[64] = {};
  if (!num_sms[dev] &&
      cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return rg_fail(PP_E_CUDA, "cannot read the SM count");
  const int grid = units < num_sms[dev] ? units : num_sms[dev];
  pp_rows_gemm_kernel<<<grid, kRgThreads, kRgSmem, st>>>(w_tiled, xs, y, (int32_t)ldy, (int32_t)n,
                                                        (int32_t)t, kchunks, tblocks, units,
                                                        accumulate ? 1 : 0, err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char msg[160];
    snprintf(msg, sizeof msg, "pp_rows_gemm launch: %s", cudaGetErrorString(e));
    return rg_fail(PP_E_CUDA, msg);
  }
  return PP_OK;
}
}  // namespace pp

extern "C" pp_status pp_rows_gemm(const uint16_t* w_tiled, uint32_t n, uint32_t k, const float* x,
                                  uint32_t t, float* y, void* work, uint64_t work_bytes,
                                  uint32_t* err, void* stream) {
  if (!w_tiled || !x || !y || !work || !err) return rg_fail(PP_E_INVALID, "null argument");
  if (n == 0 || k == 0 || t == 0 || n > (1u << 24) || k > (1u << 20) || t > (1u << 20))
    return rg_fail(PP_E_INVALID, "sizes out of range");
  if (work_bytes < pp_rows_gemm_work_bytes(t, k))
    return rg_fail(PP_E_INVALID, "work buffer smaller than pp_rows_gemm_work_bytes(t, k)");
  if ((uintptr_t)w_tiled % 16 || (uintptr_t)work % 1024)
    return rg_fail(PP_E_INVALID, "w_tiled must be 16-byte and work 1024-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const int kchunks = (int)((k + kChunkK - 1) / kChunkK);
  const int tblocks = (int)((t + kRgN - 1) / kRgN);
  const int64_t sunits = (int64_t)tblocks * kRgN * kchunks * 8;
  const int sgrid = (int)((sunits + 255) / 256 < 4096 ? (sunits + 255) / 256 : 4096);
  pp_rows_split_kernel<<<sgrid, 256, 0, st>>>(x, (int32_t)k, (int32_t)t, (int32_t)k, kchunks,
                                              tblocks, (uint8_t*)work);
  return rows_gemm_blocks(w_tiled, n, k, (const uint8_t*)work, t, y, n, false, err, st);
}
