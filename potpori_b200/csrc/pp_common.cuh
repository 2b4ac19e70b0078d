// Shared device helpers for the sm_100a verify-pass kernels: BF16 decode, packed F32x2 FMA,
// mbarrier + TMA wrappers (plain, non-multicast loads only), programmatic dependent launch
// controls and the bounded waits every kernel uses.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pp {

// Host: message of the last failure of an entry point without a handle (pp_last_error(NULL)).
void set_global_error(const char* msg);

// ---- limits and layout constants -------------------------------------------------------
constexpr int kMaxRows = 16;        // largest chunk (rows of the activation) a launch takes
constexpr int kTileRows = 128;      // GEMV output rows per tile (= one head of 128 for QKV)
constexpr int kChunkK = 64;         // K columns per pipeline stage (128 B of BF16)
constexpr int kConsumerWarps = 8;   // GEMV math warps; one more warp issues TMA
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kAttnTile = 32;       // keys per attention tile
constexpr int kAttnThreads = 256;
constexpr int kMaxHeadDim = 128;   // widest attention head the kernels take

// Bounded-wait budget: every spin on an mbarrier or a counter gives up after this many
// polls (far beyond any legitimate wait, which ends in microseconds), records ST_TIMEOUT in
// the step status word and returns.
constexpr uint32_t kSpinLimit = 1u << 22;

// Status bits written to StepResult::status by the kernels.
enum : int32_t {
  ST_BAD_STEP = 1,       // pos/m outside [0, capacity) or the chunk limits
  ST_NONFINITE_IN = 2,   // a non-finite value in the hidden input
  ST_TIMEOUT = 4,        // a bounded wait expired
  ST_NONFINITE_OUT = 8,  // non-finite logits in some row
};

// Per-step inputs, resident in device memory so captured graphs stay position independent.
struct StepDesc {
  int32_t pos;
  int32_t m;
  int32_t n_drafts;
  int32_t flags;  // bit 0: write full logits
  int32_t tokens[kMaxRows];
  int32_t drafts[kMaxRows];
};

// Per-step results of the tail (argmax, top-2, accept/mismatch) and the status word.
struct StepResult {
  int32_t argmax[kMaxRows];
  float top1[kMaxRows];
  float top2[kMaxRows];
  int32_t nonfinite_rows;  // bit r set when row r had a non-finite logit
  int32_t n_accepted;
  int32_t correction;
  int32_t status;
};

// A malformed step header (one that did not come through the host checks) makes every
// kernel of the step return before touching memory; pp_step_begin_kernel reports it.
__device__ __forceinline__ bool bad_step(const StepDesc* d, int32_t capacity, int32_t max_rows) {
  const int32_t pos = d->pos, m = d->m;
  return pos < 0 || m < 1 || m > max_rows || (int64_t)pos + m > capacity;
}

// ---- scalar helpers ---------------------------------------------------------------------
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

// d += a * b on two F32 lanes with one sm_100 FFMA2 instruction (IEEE fma per lane).
__device__ __forceinline__ void ffma2(float2& d, float2 a, float2 b) { d = __ffma2_rn(a, b, d); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- programmatic dependent launch -------------------------------------------------------
// Everything a kernel does before pdl_wait() may only touch read-only data (weights,
// tables). pdl_wait() returns once the previous kernel in the stream has completed and its
// writes are visible.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- mbarrier -------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
// Counter increment that publishes this CTA's earlier global writes (release, cumulative over
// the writes of the threads that met thread 0 at the preceding CTA barrier) and observes those
// of the CTAs that incremented before it (acquire).
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false when the phase did not complete within kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Rows of the split activation block: the MMA's N dimension (8, or 16 for 16-row chunks).
template <int MT>
struct SplitRows {
  static constexpr int R = MT <= 8 ? 8 : 16;
  static constexpr int kBlock = 2 * R * 128;  // bytes per 64-column chunk: [hi|lo][R][128 B]
};

// Byte offset of element (row m, column k) of a split activation matrix: for each 64-column
// chunk a block [hi, lo][R rows][64 BF16], the 16-byte unit u of row m stored at u ^ (m & 7)
// (bank-conflict-free ldmatrix). hi = bf16(v), lo = bf16(v - hi): hi + lo carries v to about
// 2^-17 relative, and the BF16 products of the MMA are exact in its F32 accumulator.
template <int MT>
__host__ __device__ __forceinline__ size_t split_offset(int m, int k, int hl) {
  constexpr int R = SplitRows<MT>::R;
  const int c = k >> 6, kk = k & 63;
  return (size_t)c * SplitRows<MT>::kBlock + (size_t)(hl * R + m) * 128 +
         ((((kk >> 3) ^ (m & 7))) << 4) + ((kk & 7) << 1);
}

__device__ __forceinline__ void split_bf16(float v, uint16_t& hi, uint16_t& lo) {
  hi = f32_to_bf16_rne(v);
  lo = f32_to_bf16_rne(v - __uint_as_float((uint32_t)hi << 16));
}

template <int MT>
__device__ __forceinline__ void store_split(uint8_t* base, int m, int k, float v) {
  uint16_t hi, lo;
  split_bf16(v, hi, lo);
  *(uint16_t*)(base + split_offset<MT>(m, k, 0)) = hi;
  *(uint16_t*)(base + split_offset<MT>(m, k, 1)) = lo;
}

// ---- KV cache layout -----------------------------------------------------------------------
// The cache holds, per layer and KV head, one row per position: the F32 key (value) vector
// stored as two BF16 parts, hi = bf16(x) and lo = bf16(x - hi) (x = hi + lo to about 2^-17
// relative), so the attention kernel feeds it to the tensor cores without a conversion pass.
// Row j = [hi: hdk BF16][lo: hdk BF16], hdk = head_dim rounded up to the MMA K step (16),
// padding zero; within each part the 16-byte unit u (dims 8u..8u+7) sits at u ^ (j & mask),
// mask = min(hdk / 8, 8) - 1, so ldmatrix reads of 8 consecutive rows hit 8 bank groups.
// A 32-position tile of one head is a contiguous block (one bulk copy).
__host__ __device__ __forceinline__ int kv_hdk(int hd) { return (hd + 15) & ~15; }
__host__ __device__ __forceinline__ int kv_row_bytes(int hd) { return 4 * kv_hdk(hd); }
__host__ __device__ __forceinline__ int kv_swz_mask(int hd) {
  const int u = kv_hdk(hd) >> 3;
  return (u < 8 ? u : 8) - 1;
}
// Byte offset of (dim d, part 0 = hi / 1 = lo) inside row j.
__host__ __device__ __forceinline__ int kv_offset(int j, int d, int part, int hd) {
  return part * 2 * kv_hdk(hd) + ((((d >> 3) ^ (j & kv_swz_mask(hd)))) << 4) + ((d & 7) << 1);
}

// Writes v as the (hi, lo) parts of dim d of cache row `row` (row j of its head).
__device__ __forceinline__ void kv_store(uint8_t* row, int j, int d, int hd, float v) {
  uint16_t hi, lo;
  split_bf16(v, hi, lo);
  *(uint16_t*)(row + kv_offset(j, d, 0, hd)) = hi;
  *(uint16_t*)(row + kv_offset(j, d, 1, hd)) = lo;
}

// ---- weight layout ------------------------------------------------------------------------
// Matrices are stored as the shared-memory image of the GEMV's pipeline stages: for tile t
// (128 output rows) and K chunk c (64 columns), one contiguous 16 KB block of 128 rows x
// 128 bytes in which the 16-byte unit u of row r sits at position u ^ (r & 7) (the 128-byte
// swizzle, so the consumers' row reads are bank-conflict free). Blocks are ordered tile-major,
// which is the stream-K iteration order: every CTA streams one contiguous range of bytes.
// Element offset of (row n, column k) with kchunks 64-column chunks per row:
__host__ __device__ __forceinline__ int64_t tiled_offset(int64_t n, int64_t k, int64_t kchunks) {
  const int64_t t = n >> 7, r = n & 127, c = k >> 6, kk = k & 63;
  return (((t * kchunks + c) * 128 + r) << 6) + ((((kk >> 3) ^ (r & 7))) << 3) + (kk & 7);
}

// One contiguous global -> shared copy on the bulk-copy (TMA) engine, completing on `bar`.
// 16-byte aligned addresses, size a multiple of 16. Destination is this CTA's own memory.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- TMA (tiled, no multicast) ------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---- named barrier among the consumer warps ----------------------------------------------
// Barrier over `count` threads (a multiple of 32) on named barrier `id`.
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

}  // namespace pp
