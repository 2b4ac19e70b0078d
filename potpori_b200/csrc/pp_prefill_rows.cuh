// Row kernels of the prompt prefill (pp_shard_prefill): the pieces between the tcgen05
// projections (rows_gemm_blocks) when a whole prompt chunk of t rows goes through the layers
// at once. Rows are F32 with a row stride equal to their width; the inputs of the projections
// are written straight into their BF16 hi + lo activation blocks (pp_rows_blocks.cuh), and
// the residual adds happen in the projections' epilogues. The arithmetic is the verify
// pass's: RMSNorm x * (1 / sqrt(mean(x^2) + eps)) * w (tiny.rs:20-23), per-head QK-norm and
// rotate-half RoPE at the absolute position with the K/V rows written into the cache
// (model.rs:267-302, tiny.rs:24-37), SwiGLU g / (1 + e^-g) * u (tiny.rs:111-115).
#pragma once
#include "pp_attn.cuh"
#include "pp_common.cuh"
#include "pp_rows_blocks.cuh"

namespace pp {

// x[t][c] = embedding row of tokens[t] (BF16 decoded), c < h; grid (t), 256 threads.
__global__ void pp_pre_embed_kernel(const uint16_t* table, int32_t kchunks, const int32_t* tokens,
                                 int32_t h, float* x) {
  const int t = blockIdx.x, tok = tokens[t];
  for (int c = threadIdx.x; c < h; c += blockDim.x)
    x[(size_t)t * h + c] = __uint_as_float((uint32_t)table[tiled_offset(tok, c, kchunks)] << 16);
}

// RMSNorm of row t, x[t][c] * (1 / sqrt(mean_c x[t][c]^2 + eps)) * w[c], written straight
// into the projection's activation blocks (kchunks 64-column chunks, columns past h zero);
// grid (t), 256 threads.
__global__ void pp_pre_norm_split_kernel(const float* x, const float* w, int32_t h, float eps,
                                      int32_t kchunks, uint8_t* xs) {
  __shared__ float red[8];
  const float* xr = x + (size_t)blockIdx.x * h;
  float ss = 0.f;
  for (int c = threadIdx.x; c < h; c += blockDim.x) ss += xr[c] * xr[c];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += red[i];
  const float rinv = 1.0f / sqrtf(tot / (float)h + eps);
  for (int u = threadIdx.x; u < kchunks * 8; u += blockDim.x) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int c = 8 * u + e;
      v[e] = c < h ? xr[c] * rinv * w[c] : 0.f;
    }
    rows_store_unit(xs, kchunks, (int)blockIdx.x, u, v);
  }
}

// Projections qkv[t][Q + 2 KV] of rows at positions pos + t: per head RMSNorm with q_norm /
// k_norm and RoPE, queries to q[t][Q], keys and values into the cache rows of their heads.
// Head size 128 (hd is checked by the caller). Grid (t, ceil((n_heads + 2 n_kv) / 4)), 256
// threads: four heads per block, 64 threads per head, one per dim pair (i, i + 64).
__global__ void __launch_bounds__(256)
    pp_pre_qkv_kernel(const float* qkv, int32_t t_rows, int32_t pos, int32_t nh, int32_t nkv,
                   int32_t hd, float eps, const float* qn, const float* kn, const float2* rope,
                   uint8_t* kc, uint8_t* vc, int32_t capacity, float* q) {
  constexpr int HD = 128, HALF = 64;
  __shared__ float red[8];
  const int t = blockIdx.x, i = threadIdx.x & (HALF - 1), hl = threadIdx.x / HALF;
  const int head = blockIdx.y * 4 + hl;
  const int Q = nh * HD, KV = nkv * HD;
  const bool valid = head < nh + 2 * nkv;
  const float* src = qkv + (size_t)t * (Q + 2 * KV) + (size_t)head * HD;
  const int p = pos + t;
  const float x0 = valid ? src[i] : 0.f, x1 = valid ? src[i + HALF] : 0.f;
  const float ss_w = warp_sum(x0 * x0 + x1 * x1);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss_w;
  __syncthreads();
  if (!valid) return;
  if (head >= nh + nkv) {  // value row
    uint8_t* row = vc + ((size_t)(head - nh - nkv) * capacity + p) * kv_row_bytes(HD);
    kv_store(row, p, i, HD, x0);
    kv_store(row, p, i + HALF, HD, x1);
    return;
  }
  const float ss = red[2 * hl] + red[2 * hl + 1];
  const float rms = sqrtf(ss / (float)HD + eps);
  const bool isq = head < nh;
  const float* w = isq ? qn : kn;
  const float y0 = x0 / rms * w[i], y1 = x1 / rms * w[i + HALF];
  const float2 cs = rope[(size_t)p * HALF + i];
  const float o0 = y0 * cs.x - y1 * cs.y, o1 = y1 * cs.x + y0 * cs.y;
  if (isq) {
    float* dst = q + (size_t)t * Q + (size_t)head * HD;
    dst[i] = o0;
    dst[i + HALF] = o1;
  } else {
    uint8_t* row = kc + ((size_t)(head - nh) * capacity + p) * kv_row_bytes(HD);
    kv_store(row, p, i, HD, o0);
    kv_store(row, p, i + HALF, HD, o1);
  }
}

// SwiGLU over the packed gate/up output (64-row blocks: gate rows then up rows of each 128),
// act[t][j] = g / (1 + e^-g) * u for j < I, written straight into the down projection's
// activation blocks (kchunks 64-column chunks, columns past I zero); one thread per row and 8
// columns, grid-stride.
__global__ void pp_pre_swiglu_split_kernel(const float* gu, int32_t gu_rows, int32_t I,
                                        int32_t t_rows, int32_t kchunks, uint8_t* xs) {
  const int64_t per_row = (int64_t)kchunks * 8, n = (int64_t)t_rows * per_row;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(e / per_row), u = (int)(e - row * per_row);
    const float* src = gu + (size_t)row * gu_rows;
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = 8 * u + q;
      float a = 0.f;
      if (j < I) {
        const int pg = (j >> 6) * 128 + (j & 63);
        const float g = src[pg], up = src[pg + 64];
        a = g / (1.0f + expf(-g)) * up;
      }
      v[q] = a;
    }
    rows_store_unit(xs, kchunks, row, u, v);
  }
}

// ---- causal attention of a prompt chunk ---------------------------------------------------
// Flash-style: one CTA per (KV head h, block of BQ = 16 NW / G prompt rows), NW warps, warp w
// the 16 rows r0..r0+15 of query head h G + g. The query fragments stay in registers, the 32-key
// K/V tiles of the cache stream through a ring of bulk copies, and per tile a warp computes
// S = Q K^T (16 x 32) on the tensor cores, the online softmax of its rows in registers
// (running max, rescale, running sum), and O += P V with P taken straight from the S
// accumulators. Every F32 operand is carried as hi + lo BF16 with the three products
// hi.hi + hi.lo + lo.hi, as in the verify pass's attention; scores are divided by
// sqrt(head_dim) and row r sees keys 0..pos + r (tiny.rs:77-101). The normalised row r, columns
// (h G + g) 128 + d, goes straight into the O projection's activation blocks xs (q_dim / 64
// chunks). Head size 128, G <= NW; grid
// (n_kv, ceil(t / BQ)), 32 NW threads, flash_smem_bytes(NW, NS) of dynamic shared memory
// (NS K/V tiles in flight).
constexpr int kFlashHd = 128;
constexpr int kFlashRowB = 4 * kFlashHd;  // a cache row: hi and lo parts of 128 dims
constexpr int kFlashTileB = kAttnTile * kFlashRowB;  // one K (or V) tile
__host__ __device__ constexpr size_t flash_smem_bytes(int nw, int ns) {
  return (size_t)ns * 2 * kFlashTileB + 16 * nw * (size_t)kFlashRowB + 8 * ns + 128;
}

__device__ __forceinline__ uint32_t pack_bf16x2(uint16_t lo_half, uint16_t hi_half) {
  return (uint32_t)lo_half | ((uint32_t)hi_half << 16);
}
// (a, b) as the hi and lo BF16x2 words of an MMA fragment register (a in the low half).
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  uint16_t ah, al, bh, bl;
  split_bf16(a, ah, al);
  split_bf16(b, bh, bl);
  hi = pack_bf16x2(ah, bh);
  lo = pack_bf16x2(al, bl);
}

template <int NW, int NS>
__global__ void __launch_bounds__(32 * NW, 256 / (32 * NW))
    pp_pre_flash_kernel(const float* q, const uint8_t* kc, const uint8_t* vc, int32_t capacity,
                     int32_t nh, int32_t nkv, int32_t pos, int32_t t, float scale,
                     uint8_t* xs, StepResult* res) {
  constexpr int HD = kFlashHd, RB = kFlashRowB, TB = kFlashTileB, NT = 32 * NW, NQ = 16 * NW;
  extern __shared__ uint8_t flash_smem_raw[];
  uint8_t* ring = (uint8_t*)(((uintptr_t)flash_smem_raw + 127) & ~(uintptr_t)127);
  uint8_t* qsm = ring + (size_t)NS * 2 * TB;
  uint64_t* full = (uint64_t*)(qsm + NQ * RB);

  const int G = nh / nkv, BQ = NQ / G, wpg = BQ / 16;
  const int h = blockIdx.x, b = gridDim.y - 1 - blockIdx.y;  // the longest blocks start first
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g4 = lane >> 2, t4 = lane & 3;
  const int g = warp / wpg, r0 = b * BQ + (warp - g * wpg) * 16;
  const int Q = nh * HD;
  const int kend = min(pos + t, pos + b * BQ + BQ);  // keys visible to the block's last row
  const int ntiles = (kend + kAttnTile - 1) / kAttnTile;
  const float inv_scale = 1.0f / scale;
  const uint8_t* kb = kc + (size_t)h * capacity * RB;
  const uint8_t* vb = vc + (size_t)h * capacity * RB;

  auto issue = [&](int tile) {
    const int bi = tile % NS, j0 = tile * kAttnTile;
    const uint32_t bytes = (uint32_t)min(kAttnTile, kend - j0) * RB;
    uint8_t* dst = ring + (size_t)bi * 2 * TB;
    mbar_arrive_expect_tx(&full[bi], 2 * bytes);
    bulk_load(dst, kb + (size_t)j0 * RB, bytes, &full[bi]);
    bulk_load(dst + TB, vb + (size_t)j0 * RB, bytes, &full[bi]);
  };
  if (tid == 0) {
    for (int i = 0; i < NS; ++i) mbar_init(&full[i], 1);
    fence_barrier_init();
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int i = 0; i < NS && i < ntiles; ++i) issue(i);
  }

  // The block's query vectors (qi = 16 w + i: warp w's row i) as hi/lo rows in the cache-row
  // layout; rows past the chunk are zero.
  for (int e = tid; e < NQ * (HD / 8); e += NT) {
    const int qi = e >> 4, d0 = (e & 15) * 8;
    const int w = qi >> 4, gq = w / wpg, row = b * BQ + (w - gq * wpg) * 16 + (qi & 15);
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (row < t) {
      const float4* src = (const float4*)(q + (size_t)row * Q + (size_t)(h * G + gq) * HD + d0);
      const float4 x0 = src[0], x1 = src[1];
      v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
      v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
    }
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) split_pair(v[2 * k], v[2 * k + 1], hw[k], lw[k]);
    uint8_t* row_p = qsm + (size_t)qi * RB;
    *(uint4*)(row_p + kv_offset(qi, d0, 0, HD)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *(uint4*)(row_p + kv_offset(qi, d0, 1, HD)) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
  __syncthreads();
  uint32_t qa[HD / 16][2][4];  // [k step][hi, lo] A fragments of the warp's 16 rows
  {
    const int qrow = warp * 16 + (lane & 15);
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      const uint8_t* qp = qsm + (size_t)qrow * RB + (((2 * ks + (lane >> 4)) ^ (qrow & 7)) << 4);
      ldmatrix_x4a(qa[ks][0], qp);
      ldmatrix_x4a(qa[ks][1], qp + 2 * HD);
    }
  }
  // Last key of each of the thread's two rows (g4 and g4 + 8), and of the warp.
  const int limA = min(pos + r0 + g4, kend - 1), limB = min(pos + r0 + g4 + 8, kend - 1);
  const int wlim = min(pos + r0 + 15, kend - 1);

  float o[HD / 8][4];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  int tile = 0;
  for (; tile < ntiles; ++tile) {
    const int bi = tile % NS, j0 = tile * kAttnTile;
    const int nrows = min(kAttnTile, kend - j0);
    const uint8_t* kt = ring + (size_t)bi * 2 * TB;
    uint8_t* vt = ring + (size_t)bi * 2 * TB + TB;
    // V rows past the keys are zeroed (P is 0 there, and 0 * stale bits must be 0).
    for (int e = nrows * RB / 16 + tid; e < TB / 16; e += NT)
      ((uint4*)vt)[e] = make_uint4(0u, 0u, 0u, 0u);
    const bool got = mbar_wait(&full[bi], (uint32_t)(tile / NS) & 1u);
    if (__syncthreads_or(!got)) break;
    if (j0 <= wlim) {
      float s[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          const int krow = 16 * np + (lane & 7) + ((lane >> 4) << 3);
          const int u = 2 * ks + ((lane >> 3) & 1);
          const uint8_t* kp = kt + (size_t)krow * RB + ((u ^ (krow & 7)) << 4);
          uint32_t kh[4], kl[4];
          ldmatrix_x4a(kh, kp);
          ldmatrix_x4a(kl, kp + 2 * HD);
          mma_bf16_16816(s[2 * np], qa[ks][0], kh[0], kh[1]);
          mma_bf16_16816(s[2 * np], qa[ks][0], kl[0], kl[1]);
          mma_bf16_16816(s[2 * np], qa[ks][1], kh[0], kh[1]);
          mma_bf16_16816(s[2 * np + 1], qa[ks][0], kh[2], kh[3]);
          mma_bf16_16816(s[2 * np + 1], qa[ks][0], kl[2], kl[3]);
          mma_bf16_16816(s[2 * np + 1], qa[ks][1], kh[2], kh[3]);
        }
      }
      // Scale, causal mask, online softmax of rows g4 (elements 0, 1) and g4 + 8 (2, 3).
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = j0 + 8 * j + 2 * t4 + (e & 1);
          const float v = key <= (e < 2 ? limA : limB) ? s[j][e] * inv_scale : -INFINITY;
          s[j][e] = v;
          mx[e >> 1] = fmaxf(mx[e >> 1], v);
        }
      float alpha[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
        mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
        const float mn = fmaxf(mrow[i], mx[i]);
        alpha[i] = (mrow[i] == -INFINITY) ? 0.f : __expf(mrow[i] - mn);
        mrow[i] = mn;
        lrow[i] *= alpha[i];
      }
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
        o[n][0] *= alpha[0];
        o[n][1] *= alpha[0];
        o[n][2] *= alpha[1];
        o[n][3] *= alpha[1];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p = (s[j][e] == -INFINITY) ? 0.f : __expf(s[j][e] - mrow[e >> 1]);
          s[j][e] = p;
          lrow[e >> 1] += p;
        }
      // O += P V: P's A fragments are the S accumulators of key tiles 2 ks and 2 ks + 1.
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        uint32_t ph[4], pl[4];
        split_pair(s[2 * ks][0], s[2 * ks][1], ph[0], pl[0]);
        split_pair(s[2 * ks][2], s[2 * ks][3], ph[1], pl[1]);
        split_pair(s[2 * ks + 1][0], s[2 * ks + 1][1], ph[2], pl[2]);
        split_pair(s[2 * ks + 1][2], s[2 * ks + 1][3], ph[3], pl[3]);
        const int vrow = 16 * ks + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
        for (int dp = 0; dp < HD / 16; ++dp) {
          const int u = 2 * dp + (lane >> 4);
          const uint8_t* vp = vt + (size_t)vrow * RB + ((u ^ (vrow & 7)) << 4);
          uint32_t vh[4], vl[4];
          ldmatrix_x4_trans(vh, vp);
          ldmatrix_x4_trans(vl, vp + 2 * HD);
          mma_bf16_16816(o[2 * dp], ph, vh[0], vh[1]);
          mma_bf16_16816(o[2 * dp], ph, vl[0], vl[1]);
          mma_bf16_16816(o[2 * dp], pl, vh[0], vh[1]);
          mma_bf16_16816(o[2 * dp + 1], ph, vh[2], vh[3]);
          mma_bf16_16816(o[2 * dp + 1], ph, vl[2], vl[3]);
          mma_bf16_16816(o[2 * dp + 1], pl, vh[2], vh[3]);
        }
      }
    }
    __syncthreads();  // the tile's buffer is free
    if (tid == 0 && tile + NS < ntiles) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(tile + NS);
    }
  }
  if (tile < ntiles) {  // a wait expired: report, and let the copies in flight land
    if (tid == 0) {
      atomicOr(&res->status, ST_TIMEOUT);
      for (int tt = tile; tt < ntiles && tt < tile + NS; ++tt) mbar_wait(&full[tt % NS], (uint32_t)(tt / NS) & 1u);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    lrow[i] += __shfl_xor_sync(0xffffffffu, lrow[i], 1);
    lrow[i] += __shfl_xor_sync(0xffffffffu, lrow[i], 2);
  }
  const int rowA = r0 + g4, rowB = rowA + 8, kcq = Q / kChunkK;
  const int col = (h * G + g) * HD + 2 * t4;
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) {
    if (rowA < t) rows_store_pair(xs, kcq, rowA, col + 8 * n, o[n][0] / lrow[0], o[n][1] / lrow[0]);
    if (rowB < t) rows_store_pair(xs, kcq, rowB, col + 8 * n, o[n][2] / lrow[1], o[n][3] / lrow[1]);
  }
}

}  // namespace pp
