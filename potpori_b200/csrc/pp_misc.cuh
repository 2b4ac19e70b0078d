// Small kernels around the verify pass: the shard's input kernel (embedding gather or hidden
// check, and the first GEMV's normalised operand), the seeded weight generator, packing uploaded parameters into the shard's HBM layout, and fills.
#pragma once
#include "pp_common.cuh"

namespace pp {

// The shard's input rows and the operand of its first GEMV. On the first shard x is the
// embedding rows of the chunk's tokens, BF16 decoded to F32 (src/qwen/model.rs:239-241);
// otherwise x is the hidden state received from the previous shard, checked finite
// (src/qwen/model.rs:384-386). For the GEMV after it (QKV, or the vocab head of a shard with
// no layers) this writes split(x * norm_w) in the split activation layout and, per 128-column
// tile, each row's sum of squares of x into the partials [tiles][kMaxRows]; the GEMV scales
// its accumulator by 1 / sqrt(mean(x^2) + eps), the RMSNorm of src/qwen/tiny.rs:20-23.
// Grid (ceil(hidden / 128), MT), one thread per column; rows past m are left alone.
struct PrepArgs {
  const uint16_t* table;  // embedding (first shard) or NULL (hidden input in x)
  int32_t hidden, kchunks, vocab;
  float* x;
  int32_t ldx;
  const float* norm_w;  // norm of the first GEMV; NULL: no operand to write
  uint8_t* xw;
  float* ss;
  const StepDesc* desc;
  StepResult* res;
};

// One (128-column tile, chunk row r) unit by 128 threads (t = 0..127, named barrier bar_id);
// red: 4 floats of shared memory.
template <int MT>
__device__ __forceinline__ void prep_unit(const PrepArgs& p, int tile, int r, int t, int bar_id,
                                          float* red) {
  const int n = tile * 128 + t;
  bool skip = false;
  int tok = 0;
  if (p.table) {
    tok = p.desc->tokens[r];
    if (tok < 0 || tok >= p.vocab) {
      if (tile == 0 && t == 0) atomicOr(&p.res->status, ST_BAD_STEP);
      skip = true;  // uniform over the unit
    }
  }
  float v = 0.f;
  if (!skip && n < p.hidden) {
    float* xr = p.x + (size_t)r * p.ldx;
    if (p.table) {
      v = __uint_as_float((uint32_t)p.table[tiled_offset(tok, n, p.kchunks)] << 16);
      xr[n] = v;
    } else {
      v = xr[n];
      if (!isfinite(v)) atomicOr(&p.res->status, ST_NONFINITE_IN);
    }
    if (p.norm_w) store_split<MT>(p.xw, r, n, v * p.norm_w[n]);
  }
  const float sq = warp_sum(v * v);
  if ((t & 31) == 0) red[t >> 5] = sq;
  named_sync(bar_id, 128);
  if (t == 0) p.ss[tile * kMaxRows + r] = (red[0] + red[1]) + (red[2] + red[3]);
  named_sync(bar_id, 128);  // red is free again
}

// Grid (ceil(hidden / 128), MT), 128 threads; rows past m are left alone.
template <int MT>
__global__ void __launch_bounds__(128) pp_input_prep_kernel(const PrepArgs p, int32_t capacity) {
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (bad_step(p.desc, capacity, MT)) return;
  pdl_wait();
  if ((int)blockIdx.y >= p.desc->m) return;
  __shared__ float red[4];
  prep_unit<MT>(p, blockIdx.x, blockIdx.y, threadIdx.x, 1, red);
}

// ---- seeded generator (bit-identical to the oracle's or_gen_bf16) -------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ uint16_t gen_bf16(uint64_t key, int64_t i, float scale) {
  int32_t s = 0;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const uint64_t r = mix64(key + (uint64_t)(3 * i + j + 1) * 0x9E3779B97F4A7C15ull);
    s += (int32_t)(r & 0xffff) + (int32_t)((r >> 16) & 0xffff) + (int32_t)((r >> 32) & 0xffff) +
         (int32_t)(r >> 48);
  }
  return f32_to_bf16_rne(__fmul_rn((float)(s - 393210), scale));
}

// Where logical row r of a checkpoint matrix lands in the packed matrix:
// (r / blk) * blk_stride + r % blk + offset. QKV sections use blk = rows (one block);
// gate/up are interleaved in 64-row blocks so one 128-row tile holds both halves.
struct RowMap {
  int32_t blk, blk_stride, offset;
  __host__ __device__ int64_t operator()(int64_t r) const {
    return (r / blk) * blk_stride + (r % blk) + offset;
  }
};

// Fill a [rows][cols] logical matrix from the generator into the tiled layout.
__global__ void pp_gen_matrix_kernel(uint16_t* dst, int64_t rows, int64_t cols, int64_t kchunks,
                                  RowMap map, uint64_t key, float scale) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    dst[tiled_offset(map(r), c, kchunks)] = gen_bf16(key, i, scale);
  }
}

// Copy an uploaded [rows][cols] matrix (BF16 bits, or F32 rounded to BF16 as the reference's
// loader does, src/qwen/hf.rs:248-253) into the packed layout.
__global__ void pp_pack_matrix_kernel(uint16_t* dst, const void* src, int32_t src_f32, int64_t rows,
                                   int64_t cols, int64_t kchunks, RowMap map) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const uint16_t v = src_f32 ? f32_to_bf16_rne(((const float*)src)[i]) : ((const uint16_t*)src)[i];
    dst[tiled_offset(map(r), c, kchunks)] = v;
  }
}

__global__ void pp_fill_f32_kernel(float* dst, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = v;
}

// Seeded N(0,1) values (rounded through BF16) for KV rows [0, rows) of one layer: a warm
// context for benchmarks; the oracle's or_shard_fill_kv writes the same values.
__global__ void pp_fill_kv_kernel(uint8_t* kc, uint8_t* vc, int64_t rows, int32_t kv_dim,
                               int32_t n_kv, int32_t hd, int64_t capacity, uint64_t key) {
  const int64_t n = rows * kv_dim;
  const float scale = 1.0f / 65536.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / kv_dim, col = i - row * kv_dim;
    const int64_t h = col / hd, dd = col - h * hd;
    const size_t base = ((size_t)h * capacity + row) * kv_row_bytes(hd);
    kv_store(kc + base, (int)row, (int)dd, hd, __uint_as_float((uint32_t)gen_bf16(key, 2 * i, scale) << 16));
    kv_store(vc + base, (int)row, (int)dd, hd, __uint_as_float((uint32_t)gen_bf16(key, 2 * i + 1, scale) << 16));
  }
}

}  // namespace pp
