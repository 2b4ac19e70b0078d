// Activation blocks of the tensor-core prompt projection (pp_rows_gemm): F32 rows x[t][c]
// carried as BF16 hi + lo parts in the MMA's K-major 128-byte-swizzled operand form,
// xs[tb][chunk][part][128 rows][64 columns], part 0 = hi, 1 = lo, the 16-byte unit u of row r
// at u ^ (r & 7). Shared by the projection and by the prefill's row kernels that write its
// input directly (RMSNorm + split, SwiGLU + split).
#pragma once
#include <cuda_runtime.h>

#include "../../include/potpori_b200.h"
#include "pp_common.cuh"

namespace pp {

constexpr int kRgN = 128;                      // activation rows per block (TMEM columns)
constexpr int kRgXBytes = kRgN * kChunkK * 2;  // 16 KB per activation part

// Stores the 8 values v of columns 8 u .. 8 u + 7 of activation row `row` as hi and lo units.
__device__ __forceinline__ void rows_store_unit(uint8_t* xs, int kchunks, int row, int u,
                                                const float (&v)[8]) {
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    uint16_t h0, l0, h1, l1;
    split_bf16(v[2 * e], h0, l0);
    split_bf16(v[2 * e + 1], h1, l1);
    hi[e] = (uint32_t)h0 | ((uint32_t)h1 << 16);
    lo[e] = (uint32_t)l0 | ((uint32_t)l1 << 16);
  }
  const int tb = row / kRgN, r = row % kRgN, c = u >> 3, uu = u & 7;
  uint8_t* blk = xs + ((size_t)tb * kchunks + c) * 2 * kRgXBytes;
  const size_t off = (size_t)r * 128 + (size_t)((uu ^ (r & 7)) << 4);
  *(uint4*)(blk + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  *(uint4*)(blk + kRgXBytes + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// Stores columns col and col + 1 (col even) of activation row `row` as one 32-bit word of
// each part.
__device__ __forceinline__ void rows_store_pair(uint8_t* xs, int kchunks, int row, int col,
                                                float a, float b) {
  uint16_t ah, al, bh, bl;
  split_bf16(a, ah, al);
  split_bf16(b, bh, bl);
  const int tb = row / kRgN, r = row % kRgN, c = col / kChunkK, uu = (col % kChunkK) >> 3;
  uint8_t* blk = xs + ((size_t)tb * kchunks + c) * 2 * kRgXBytes;
  const size_t off = (size_t)r * 128 + (size_t)((uu ^ (r & 7)) << 4) + (size_t)(col & 7) * 2;
  *(uint32_t*)(blk + off) = (uint32_t)ah | ((uint32_t)bh << 16);
  *(uint32_t*)(blk + kRgXBytes + off) = (uint32_t)al | ((uint32_t)bl << 16);
}

// The projection over activation rows already in block form (xs, 1024-byte aligned, rows
// 0 .. t - 1 valid): y[i][j] (row stride ldy) = sum_c W[j][c] x[i][c], or += with
// accumulate. Defined in pp_prefill.cu; checks and error text as pp_rows_gemm.
pp_status rows_gemm_blocks(const uint16_t* w_tiled, uint32_t n, uint32_t k, const uint8_t* xs,
                           uint32_t t, float* y, uint32_t ldy, bool accumulate, uint32_t* err,
                           cudaStream_t stream);

}  // namespace pp
