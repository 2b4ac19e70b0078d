// Skinny GEMV for the verify chunk: out[m][n] = sum_k W[n][k] * x[m][k] for m < M <= 8 rows of
// F32 activations against a BF16 weight matrix W[N][K] (checkpoint orientation, row-major).
//
// This is the arithmetic of the reference's `linear` (src/qwen/model.rs:166-183): F32
// products of BF16-decoded weights, summed in F32. It is HBM bound (about M flops per weight
// byte), so the kernel is organised around streaming every weight byte exactly once:
//
//  * Stream-K over the GPU. The (tile of 128 output rows) x (64-column K chunk) iteration
//    space is cut into one contiguous, equal range per CTA, so all 148 SMs get the same
//    number of weight bytes whatever N and K are. A tile split between CTAs is finished
//    by the last contributor, which sums the partial results in K order (deterministic).
//  * One producer warp streams [128 x 64] BF16 weight blocks (16 KB, stored pre-swizzled in
//    HBM in stream order) into a ring of shared-memory stages with 1-D bulk copies (TMA
//    engine, no multicast) and mbarriers; it starts before the previous kernel has finished
//    (programmatic dependent launch), since weights do not depend on it.
//  * Eight consumer warps, 16 weight rows each, on the tensor cores: the activation is
//    carried as two BF16 parts (x = hi + lo, about 2^-17 relative), so D += W.hi + W.lo with
//    m16n8k16 MMAs into F32 accumulators reproduces the F32 products of BF16 weights (the
//    CUDA-core FFMA roof is about the HBM roof at M = 8, which this sidesteps).
//  * x is either resident in shared memory for the whole K (the input RMSNorm is applied
//    while staging it, src/qwen/tiny.rs:20-23) or streamed next to the weights as split
//    blocks that the producing kernel wrote in the MMA's operand layout.
//  * Fused epilogues: QK-RMSNorm + RoPE + KV write (QKV), residual add (O, down), SwiGLU
//    (gate/up interleaved in 64-row blocks), and argmax/top-2/accept for the vocab head.
#pragma once
#include "pp_common.cuh"

namespace pp {

enum XMode : int { X_RESIDENT_NORM = 0, X_STREAM = 1 };
enum Epi : int { EPI_QKV = 0, EPI_RESADD = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3, EPI_STORE = 4 };

struct ArgRec {
  float best;
  int32_t idx;
  float second;
  int32_t nonfinite;
};

struct GemvArgs {
  const uint16_t* w;       // tiled weights (tiled_offset layout)
  const uint8_t* xsplit;   // streamed activations, split BF16 blocks (split_offset layout)
  uint8_t* out_split;      // SwiGLU output in the same split layout (input of the down GEMV)
  int32_t n_out;     // valid output columns (after the SwiGLU pairing: intermediate)
  int32_t n_packed;  // rows of the packed weight matrix
  int32_t k;         // valid K
  int32_t kp;        // padded K (multiple of 64): row stride of W and x
  int32_t tiles;     // ceil(n_packed / 128)
  int32_t kchunks;   // kp / 64
  int32_t nstages;
  // resident x
  const float* x;
  int32_t ldx;
  const float* norm_w;
  float eps;
  int32_t check_input;  // flag non-finite x values (the shard's hidden input)
  // output
  float* out;
  int32_t ldo;
  // QKV epilogue
  const float* qn;
  const float* kn;
  const float2* rope;  // [capacity][head_dim/2] (cos, sin)
  uint8_t* kcache;     // [n_kv][capacity] rows of kv_row_bytes (split BF16, kv_offset layout)
  uint8_t* vcache;
  int32_t q_dim, kv_dim, head_dim, capacity;
  // argmax epilogue
  float* logits;  // [M][vocab] when requested by the step flags
  // scratch
  float* partials;      // [grid][2][128][MT]
  uint32_t* tile_cnt;   // [tiles], zero between launches
  ArgRec* recs;         // [grid][MT]
  uint32_t* done_cnt;   // zero between launches
  const StepDesc* desc;  // step header; NULL for a standalone GEMV (m_rows gives the rows)
  StepResult* res;       // step result / status; may be NULL for a standalone GEMV
  int32_t* status;       // standalone GEMV (res NULL): where the status bits go, or NULL
  int32_t m_rows;
  // Streamed normalised input: the operand is split(x * w_norm) and the sums of squares of
  // x come as per-tile partials [ss_tiles][kMaxRows]; the accumulator is scaled by
  // 1 / sqrt(mean(x^2) + eps) (NULL ss_in: no scaling).
  const float* ss_in;
  int32_t ss_tiles;
  // Residual-add epilogue extras: also write split(x_new * wnext) for the next norm's GEMV
  // and this tile's per-row sum of squares of x_new (NULL: not needed).
  uint8_t* xw_out;
  const float* wnext;
  float* ss_out;
};

template <int MT, int XM>
struct GemvSmem {
  static constexpr int kWBytes = kTileRows * kChunkK * 2;  // 16 KB per stage
  static constexpr int kXBytes = (XM == X_STREAM) ? SplitRows<MT>::kBlock : 0;
  static __host__ __device__ size_t x_off(int ns) { return (size_t)ns * kWBytes; }
  static __host__ __device__ size_t xs_off(int ns) { return x_off(ns) + (size_t)ns * kXBytes; }
  static __host__ __device__ size_t tile_off(int ns, int kp) {
    return xs_off(ns) +
           (XM == X_RESIDENT_NORM ? (size_t)(kp / kChunkK) * SplitRows<MT>::kBlock : 0);
  }
  static __host__ __device__ size_t bar_off(int ns, int kp) {
    return tile_off(ns, kp) + (size_t)kTileRows * MT * 4;
  }
  static __host__ __device__ size_t misc_off(int ns, int kp) { return bar_off(ns, kp) + 16 * ns; }
  static __host__ __device__ size_t total(int ns, int kp) { return misc_off(ns, kp) + 512 + 1024; }
};

// Stream-K ranges in 32-bit arithmetic (T * G < 2^32: T <= 2^23 iterations, G <= 256 CTAs).
constexpr int kMaxFixup = 256;  // contributors of one split tile are at most G
__device__ __forceinline__ int sk_start(uint32_t b, uint32_t T, uint32_t G) {
  return (int)(b * T / G);
}
__device__ __forceinline__ int sk_owner(uint32_t i, uint32_t T, uint32_t G) {
  return (int)(((i + 1) * G + T - 1) / T) - 1;
}

// Records status bits (ST_*) of a launch: in the step result, or in the standalone status word.
__device__ __forceinline__ void gemv_flag(const GemvArgs& a, int32_t bits) {
  if (a.res)
    atomicOr(&a.res->status, bits);
  else if (a.status)
    atomicOr(a.status, bits);
}

__device__ __forceinline__ void argrec_merge(float& b1, int32_t& i1, float& s1, float b2,
                                             int32_t i2, float s2) {
  if (b2 > b1 || (b2 == b1 && i2 < i1)) {
    s1 = fmaxf(fmaxf(b1, s1), s2);
    b1 = b2;
    i1 = i2;
  } else {
    s1 = fmaxf(fmaxf(b2, s1), s2);
  }
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// D[16 x 8] += A[16 x 16] . B[16 x 8], BF16 inputs, F32 accumulate.
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Consumer side of the stage ring: the next stage and its parity. It persists across the
// GEMVs that share one ring (the persistent step kernel runs many in a row).
struct RingPos {
  int s;
  uint32_t phase;
};

// Shared-memory pieces of one GEMV CTA.
struct GemvShared {
  uint8_t* wst;     // weight stages [ns][16 KB]
  uint8_t* xst;     // streamed activation stages [ns][split block]
  uint8_t* xs;      // resident activation (X_RESIDENT_NORM): [kchunks][split block]
  float* tile_out;  // [128][MT]
  uint64_t* full;   // [ns], one arrival (producer) + transaction bytes
  uint64_t* empty;  // [ns], one arrival per consumer warp
  int32_t* misc;    // [0] fixup flag, [1] status bits, [8..] argmax running state (4 x MT)
  int ns;
};

// The eight consumer warps of one GEMV over this CTA's stream-K range (CTA `bid` of `G`):
// stages are taken from the ring at `rp` (advanced on return), the MMAs accumulate each tile
// segment, split tiles are finished by their last contributor, and the epilogue EPI runs on
// every finished tile. The caller has made the activation inputs visible (PDL wait or grid
// barrier). Returns false when a bounded wait expired (ST_TIMEOUT is set).
template <int MT, int XM, int EPI>
__device__ __forceinline__ bool gemv_consume(const GemvArgs& a, const GemvShared& sh, RingPos& rp,
                                             uint32_t G, uint32_t bid) {
  using L = GemvSmem<MT, XM>;
  constexpr int R = SplitRows<MT>::R;
  constexpr int NB = R / 8;  // 8-row MMA column blocks
  constexpr int XB = SplitRows<MT>::kBlock;
  const int ns = sh.ns;
  uint8_t* wst = sh.wst;
  uint8_t* xst = sh.xst;
  uint8_t* xs = sh.xs;
  float* tile_out = sh.tile_out;
  uint64_t* full = sh.full;
  uint64_t* empty = sh.empty;
  int32_t* misc = sh.misc;
  float* st_best = (float*)(misc + 8);
  int32_t* st_idx = misc + 8 + MT;
  float* st_second = (float*)(misc + 8 + 2 * MT);
  int32_t* st_nonf = misc + 8 + 3 * MT;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const uint32_t T = (uint32_t)a.tiles * (uint32_t)a.kchunks;
  const int i0 = sk_start(bid, T, G), i1 = sk_start(bid + 1, T, G);
  const int first_tile = (int)(i0 / a.kchunks);
  if (tid == 0) {
    misc[0] = 0;
    misc[1] = 0;
  }
  if (EPI == EPI_ARGMAX && tid < MT) {
    st_best[tid] = -INFINITY;
    st_idx[tid] = 0x7fffffff;
    st_second[tid] = -INFINITY;
    st_nonf[tid] = 0;
  }
  const int mv = a.desc ? a.desc->m : a.m_rows;  // rows that matter: 1 <= mv <= MT
  __shared__ float scale_s[MT];
  // RMSNorm scale of each row (tiny.rs:20-23) from the per-tile sums of squares: warp m
  // reads row m's partials with one load per lane and reduces them in a fixed tree.
  for (int m = warp; m < MT; m += kConsumerWarps) {
    float sc = 1.0f;
    if (a.ss_in && m < mv) {
      float t = 0.f;
      for (int q = lane; q < a.ss_tiles; q += 32) t += __ldcg(a.ss_in + q * kMaxRows + m);
      t = warp_sum(t);
      sc = 1.0f / sqrtf(t / (float)a.k + a.eps);
    }
    if (lane == 0) scale_s[m] = sc;
  }
  // QKV epilogue constants (q_norm, k_norm, the RoPE rows of this step's positions), staged
  // while the first weight stages are in flight.
  constexpr int kQkvHd = EPI == EPI_QKV ? kMaxHeadDim : 1;
  __shared__ float qkn_s[2][kQkvHd];
  __shared__ float2 rope_s[EPI == EPI_QKV ? MT : 1][kQkvHd / 2 > 0 ? kQkvHd / 2 : 1];
  if (EPI == EPI_QKV) {
    const int hd = a.head_dim, half = hd >> 1;
    for (int e = tid; e < 2 * hd; e += kConsumerWarps * 32)
      qkn_s[e / hd][e % hd] = e < hd ? a.qn[e] : a.kn[e - hd];
    for (int e = tid; e < mv * half; e += kConsumerWarps * 32) {
      const int m = e / half, i = e - m * half;
      rope_s[m][i] = a.rope[(size_t)(a.desc->pos + m) * half + i];
    }
  }
  consumer_sync();

  if (XM == X_RESIDENT_NORM) {
    // RMSNorm (tiny.rs:20-23): x * (1 / sqrt(mean(x^2) + eps)) * w, staged for the whole K
    // as split BF16 blocks (hi, lo) in the MMA's B-operand layout.
    __shared__ float red[kConsumerWarps][MT];
    __shared__ float inv_s[MT];
    const int k4 = a.k >> 2;
    float ss[MT];
    int bad = 0;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      ss[m] = 0.f;
      if (m < mv) {
        const float4* xr = (const float4*)(a.x + (size_t)m * a.ldx);
        for (int q = tid; q < k4; q += kConsumerWarps * 32) {
          const float4 v = xr[q];
          bad |= !(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w));
          ss[m] += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float w = warp_sum(ss[m]);
      if (lane == 0) red[warp][m] = w;
    }
    if (a.check_input && bad) atomicOr(&misc[1], ST_NONFINITE_IN);
    consumer_sync();
    if (tid < MT) {
      float t = 0.f;
      for (int w = 0; w < kConsumerWarps; ++w) t += red[w][tid];
      inv_s[tid] = 1.0f / sqrtf(t / (float)a.k + a.eps);
    }
    consumer_sync();
    // One thread per (chunk, row, 16-byte unit): 8 columns -> 8 hi + 8 lo BF16.
    const int units = a.kchunks * R * 8;
    for (int e = tid; e < units; e += kConsumerWarps * 32) {
      const int u = e & 7, m = (e >> 3) % R, c = (e >> 3) / R;
      const int k0 = c * 64 + u * 8;
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
      if (m < mv) {
        const float inv = inv_s[m];
        const float* xr = a.x + (size_t)m * a.ldx;
        if (k0 + 8 <= a.k) {
          const float4 x0 = *(const float4*)(xr + k0), x1 = *(const float4*)(xr + k0 + 4);
          const float4 w0 = *(const float4*)(a.norm_w + k0), w1 = *(const float4*)(a.norm_w + k0 + 4);
          v[0] = x0.x * inv * w0.x; v[1] = x0.y * inv * w0.y; v[2] = x0.z * inv * w0.z;
          v[3] = x0.w * inv * w0.w; v[4] = x1.x * inv * w1.x; v[5] = x1.y * inv * w1.y;
          v[6] = x1.z * inv * w1.z; v[7] = x1.w * inv * w1.w;
        } else {
          for (int j = 0; j < 8; ++j)
            if (k0 + j < a.k) v[j] = xr[k0 + j] * inv * a.norm_w[k0 + j];
        }
      }
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint16_t h0, l0, h1, l1;
        split_bf16(v[2 * j], h0, l0);
        split_bf16(v[2 * j + 1], h1, l1);
        hw[j] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        lw[j] = (uint32_t)l0 | ((uint32_t)l1 << 16);
      }
      uint8_t* blk = xs + (size_t)c * XB + (size_t)m * 128 + ((u ^ (m & 7)) << 4);
      *(uint4*)blk = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *(uint4*)(blk + R * 128) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    consumer_sync();
    if (tid == 0 && misc[1]) gemv_flag(a, misc[1]);
  }

  // Lane roles for ldmatrix: A (weights) matrix mat = lane >> 3 covers rows (mat & 1) * 8 and
  // K half (mat >> 1); B (activations) matrix mat covers K step (mat >> 1), half (mat & 1).
  const int mat = lane >> 3, l7 = lane & 7;
  const int arow = warp * 16 + l7 + (mat & 1) * 8;
  int it = i0;
  int cs = rp.s;             // ring stage of the next iteration
  uint32_t cphase = rp.phase;  // its parity
  bool ok = true;
  int t = i0 / a.kchunks;
  while (it < i1 && ok) {
    const int tile_begin = t * a.kchunks, tile_end = tile_begin + a.kchunks;
    const int seg_begin = it, seg_end = i1 < tile_end ? i1 : tile_end;
    // Four independent accumulator chains per column block (hi/lo x even/odd K step), so
    // consecutive MMAs never wait on each other; summed at the end of the segment.
    float acc[NB][4][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int ch = 0; ch < 4; ++ch)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[nb][ch][q] = 0.f;

    for (; it < seg_end; ++it) {
      const int s = cs;
      if (!mbar_wait(&full[s], cphase)) {
        ok = false;
        break;
      }
      if (++cs == ns) {
        cs = 0;
        cphase ^= 1u;
      }
      const int c = it - tile_begin;
      const uint8_t* wb = wst + (size_t)s * L::kWBytes;
      const uint8_t* xb = (XM == X_STREAM) ? xst + (size_t)s * XB : xs + (size_t)c * XB;
      uint32_t af[4][4];
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        const int u = 2 * st + (mat >> 1);
        ldmatrix_x4(af[st], wb + arow * 128 + ((u ^ (arow & 7)) << 4));
      }
      uint32_t bh[NB][2][4], bl[NB][2][4];
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int u = 2 * (2 * p + (mat >> 1)) + (mat & 1);
          const uint8_t* row = xb + (size_t)(nb * 8 + l7) * 128 + ((u ^ l7) << 4);
          ldmatrix_x4(bh[nb][p], row);
          ldmatrix_x4(bl[nb][p], row + R * 128);
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
      for (int st = 0; st < 4; ++st)
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
          const int p = st >> 1, q = (st & 1) * 2, ch = (st & 1) * 2;
          mma_bf16(acc[nb][ch], af[st], bh[nb][p][q], bh[nb][p][q + 1]);
          mma_bf16(acc[nb][ch + 1], af[st], bl[nb][p][q], bl[nb][p][q + 1]);
        }
    }
    if (!ok) break;

    // Residual values of this tile, loaded now so that their latency overlaps the split-tile
    // handshake (only the CTA that finishes the tile uses them).
    constexpr int kPre = (kTileRows * MT + kConsumerWarps * 32 - 1) / (kConsumerWarps * 32);
    float xpre[kPre];
    if (EPI == EPI_RESADD) {
#pragma unroll
      for (int j = 0; j < kPre; ++j) {
        const int e = tid + j * kConsumerWarps * 32;
        const int m = e / kTileRows, r = e - m * kTileRows;
        const int n = t * kTileRows + r;
        xpre[j] = (e < kTileRows * MT && m < mv && n < a.n_out) ? __ldcg(a.out + (size_t)m * a.ldo + n) : 0.f;
      }
    }

    {  // accumulator fragments (x the RMSNorm scale of their row) -> tile_out[row][m]
      const int g = lane >> 2, tq = lane & 3;
      const int r0 = warp * 16 + g;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          v[q] = (acc[nb][0][q] + acc[nb][2][q]) + (acc[nb][1][q] + acc[nb][3][q]);
        const int m0 = nb * 8 + 2 * tq;
        if (m0 < MT) {
          tile_out[r0 * MT + m0] = v[0] * scale_s[m0];
          tile_out[(r0 + 8) * MT + m0] = v[2] * scale_s[m0];
        }
        if (m0 + 1 < MT) {
          tile_out[r0 * MT + m0 + 1] = v[1] * scale_s[m0 + 1];
          tile_out[(r0 + 8) * MT + m0 + 1] = v[3] * scale_s[m0 + 1];
        }
      }
    }
    consumer_sync();

    const bool whole = seg_begin == tile_begin && seg_end == tile_end;
    if (!whole) {
      // Split tile: publish this CTA's partial; the last contributor finishes the tile.
      const int slot = (t == first_tile) ? 0 : 1;
      float* mine = a.partials + ((size_t)blockIdx.x * 2 + slot) * kTileRows * MT;
      for (int e = 4 * tid; e < kTileRows * MT; e += 4 * kConsumerWarps * 32)
        *(float4*)(mine + e) = *(const float4*)(tile_out + e);
      consumer_sync();
      const int b_lo = sk_owner(tile_begin, T, G), b_hi = sk_owner(tile_end - 1, T, G);
      const int nbk = b_hi - b_lo + 1;
      if (tid == 0) {
        const uint32_t old = atom_add_acq_rel_gpu(&a.tile_cnt[t], 1u);
        misc[0] = (old == (uint32_t)(b_hi - b_lo));
      }
      // Where each contributor's partial of this tile sits (its first or its last slot).
      __shared__ int fix_off[kMaxFixup];
      for (int q = tid; q < nbk && q < kMaxFixup; q += kConsumerWarps * 32) {
        const int b = b_lo + q;
        const int bslot = (sk_start(b, T, G) / a.kchunks == t) ? 0 : 1;
        fix_off[q] = (b * 2 + bslot) * kTileRows * MT;
      }
      consumer_sync();
      if (!misc[0]) {
        ++t;
        continue;
      }
      // Sum the contributors' partials in K order. A thread owns 4 consecutive values and
      // issues the float4 loads of up to 20 contributors at once, so a tile split over 20
      // CTAs costs one L2 round trip.
      for (int e = 4 * tid; e < kTileRows * MT; e += 4 * kConsumerWarps * 32) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int b0 = 0; b0 < nbk; b0 += 20) {
          float4 pv[20];
#pragma unroll
          for (int q = 0; q < 20; ++q)
            if (b0 + q < nbk) pv[q] = __ldcg((const float4*)(a.partials + fix_off[b0 + q] + e));
#pragma unroll
          for (int q = 0; q < 20; ++q)
            if (b0 + q < nbk) {
              v.x += pv[q].x;
              v.y += pv[q].y;
              v.z += pv[q].z;
              v.w += pv[q].w;
            }
        }
        *(float4*)(tile_out + e) = v;
      }
      if (tid == 0) a.tile_cnt[t] = 0u;
      consumer_sync();
    }

    // ---------------------------------------------------------------- epilogues
    if (EPI == EPI_STORE || EPI == EPI_RESADD) {
      // Residual add (src/qwen/model.rs:318-331). With xw_out, also the next RMSNorm's
      // operand split(x_new * w) and this tile's per-row sum of squares of x_new, so the
      // next GEMV streams its input instead of normalising it in a prologue.
      const bool extras = EPI == EPI_RESADD && a.xw_out != nullptr;
      __shared__ float ssr[MT][kTileRows / 32];
#pragma unroll
      for (int j = 0; j < kPre; ++j) {
        const int e = tid + j * kConsumerWarps * 32;
        if (e >= kTileRows * MT) break;
        const int m = e / kTileRows, r = e - m * kTileRows;
        const int n = t * kTileRows + r;
        float sq = 0.f;
        if (m < mv && n < a.n_out) {
          float* o = a.out + (size_t)m * a.ldo + n;
          if (EPI == EPI_RESADD) {
            const float xn = xpre[j] + tile_out[r * MT + m];
            *o = xn;
            if (extras) {
              store_split<MT>(a.xw_out, m, n, xn * a.wnext[n]);
              sq = xn * xn;
            }
          } else {
            *o = tile_out[r * MT + m];
          }
        }
        if (extras) {  // a warp covers 32 consecutive rows of one column m
          sq = warp_sum(sq);
          if (lane == 0) ssr[m][r >> 5] = sq;
        }
      }
      if (extras) {
        consumer_sync();
        if (tid < MT) {
          float v = 0.f;
#pragma unroll
          for (int q = 0; q < kTileRows / 32; ++q) v += ssr[tid][q];
          a.ss_out[t * kMaxRows + tid] = v;
        }
      }
    } else if (EPI == EPI_SWIGLU) {
      constexpr int half = kTileRows / 2;
      for (int e = tid; e < half * MT; e += kConsumerWarps * 32) {
        const int m = e / half, r = e - m * half;
        const int n = t * half + r;
        if (m < mv && n < a.n_out) {
          const float g = tile_out[r * MT + m], u = tile_out[(r + half) * MT + m];
          store_split<MT>(a.out_split, m, n, g / (1.0f + expf(-g)) * u);  // tiny.rs:111-115
        }
      }
    } else if (EPI == EPI_QKV) {
      // Heads of this tile: per-head RMSNorm with q_norm/k_norm, rotate-half RoPE at the
      // absolute position, K and V rows written into the cache (src/qwen/model.rs:267-302,
      // tiny.rs:24-37). A warp handles one (head, row) pair.
      const int hd = a.head_dim, half = hd >> 1;
      const int heads = kTileRows / hd;
      for (int p = warp; p < heads * mv; p += kConsumerWarps) {
        const int hl = p / mv, m = p - hl * mv;
        const int n0 = t * kTileRows + hl * hd;
        const int pos = a.desc->pos + m;
        const float* v = tile_out + (size_t)(hl * hd) * MT + m;  // v[i * MT]
        if (n0 < a.q_dim + a.kv_dim) {
          const bool isq = n0 < a.q_dim;
          const float* w = qkn_s[isq ? 0 : 1];
          float ssq = 0.f;
          for (int i = lane; i < hd; i += 32) ssq += v[i * MT] * v[i * MT];
          ssq = warp_sum(ssq);
          const float rms = sqrtf(ssq / (float)hd + a.eps);
          const float2* rp = rope_s[m];
          if (isq) {
            float* dst = a.out + (size_t)m * a.ldo + n0;
            for (int i = lane; i < half; i += 32) {
              const float x0 = v[i * MT] / rms * w[i];
              const float x1 = v[(i + half) * MT] / rms * w[i + half];
              const float2 cs = rp[i];
              dst[i] = x0 * cs.x - x1 * cs.y;
              dst[i + half] = x1 * cs.x + x0 * cs.y;
            }
          } else {
            uint8_t* row = a.kcache + ((size_t)((n0 - a.q_dim) / hd) * a.capacity + pos) * kv_row_bytes(hd);
            for (int i = lane; i < half; i += 32) {
              const float x0 = v[i * MT] / rms * w[i];
              const float x1 = v[(i + half) * MT] / rms * w[i + half];
              const float2 cs = rp[i];
              kv_store(row, pos, i, hd, x0 * cs.x - x1 * cs.y);
              kv_store(row, pos, i + half, hd, x1 * cs.x + x0 * cs.y);
            }
          }
        } else if (n0 < a.q_dim + 2 * a.kv_dim) {
          uint8_t* row = a.vcache + ((size_t)((n0 - a.q_dim - a.kv_dim) / hd) * a.capacity + pos) * kv_row_bytes(hd);
          for (int i = lane; i < hd; i += 32) kv_store(row, pos, i, hd, v[i * MT]);
        }
      }
    } else if (EPI == EPI_ARGMAX) {
      // Greedy pick of src/engine.rs:14-29 over this tile's vocab rows: first index of the
      // strict maximum; any non-finite value marks the row.
      for (int m = warp; m < mv; m += kConsumerWarps) {
        float b = -INFINITY, s2 = -INFINITY;
        int32_t bi = 0x7fffffff;
        int nf = 0;
        const bool dump = a.desc->flags & 1;
        for (int r = lane; r < kTileRows; r += 32) {
          const int n = t * kTileRows + r;
          if (n >= a.n_out) break;
          const float v = tile_out[r * MT + m];
          if (dump) a.logits[(size_t)m * a.n_out + n] = v;
          if (!isfinite(v)) {
            nf = 1;
            continue;
          }
          argrec_merge(b, bi, s2, v, n, -INFINITY);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ob = __shfl_xor_sync(0xffffffffu, b, o);
          const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
          const float os = __shfl_xor_sync(0xffffffffu, s2, o);
          argrec_merge(b, bi, s2, ob, oi, os);
          nf |= __shfl_xor_sync(0xffffffffu, nf, o);
        }
        if (lane == 0) {
          argrec_merge(st_best[m], st_idx[m], st_second[m], b, bi, s2);
          st_nonf[m] |= nf;
        }
      }
    }
    consumer_sync();  // tile_out is reused by the next tile
    ++t;
  }

  rp.s = cs;
  rp.phase = cphase;
  if (!ok) {
    if (tid == 0) gemv_flag(a, ST_TIMEOUT);
    return false;
  }

  if (EPI == EPI_ARGMAX) {
    consumer_sync();
    if (tid < MT) {
      ArgRec r;
      r.best = st_best[tid];
      r.idx = st_idx[tid];
      r.second = st_second[tid];
      r.nonfinite = st_nonf[tid];
      a.recs[(size_t)blockIdx.x * MT + tid] = r;
    }
    consumer_sync();
    if (tid == 0) {
      const uint32_t old = atom_add_acq_rel_gpu(a.done_cnt, 1u);
      misc[0] = (old == (uint32_t)(G - 1));
    }
    consumer_sync();
    if (!misc[0]) return true;
    // Last CTA: reduce every CTA's record, then the accept/mismatch compare of
    // src/specdecode.rs:92-98.
    for (int m = warp; m < mv; m += kConsumerWarps) {
      float b = -INFINITY, s2 = -INFINITY;
      int32_t bi = 0x7fffffff;
      int nf = 0;
      for (uint32_t g = lane; g < G; g += 32) {
        const ArgRec* rp = a.recs + (size_t)g * MT + m;
        const float rb = __ldcg(&rp->best), rs = __ldcg(&rp->second);
        const int32_t ri = __ldcg(&rp->idx), rn = __ldcg(&rp->nonfinite);
        argrec_merge(b, bi, s2, rb, ri, rs);
        nf |= rn;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, b, o);
        const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        const float os = __shfl_xor_sync(0xffffffffu, s2, o);
        argrec_merge(b, bi, s2, ob, oi, os);
        nf |= __shfl_xor_sync(0xffffffffu, nf, o);
      }
      if (lane == 0) {
        a.res->argmax[m] = nf ? -1 : bi;
        a.res->top1[m] = b;
        a.res->top2[m] = s2;
        if (nf) {
          atomicOr(&a.res->nonfinite_rows, 1 << m);
          atomicOr(&a.res->status, ST_NONFINITE_OUT);
        }
      }
    }
    consumer_sync();
    if (tid == 0) {
      int n = 0;
      while (n < a.desc->n_drafts && n < mv && a.desc->drafts[n] == a.res->argmax[n]) ++n;
      if (n >= mv) n = mv - 1;
      a.res->n_accepted = n;
      a.res->correction = a.res->argmax[n];
      *a.done_cnt = 0u;
    }
  }
  return true;
}

template <int MT, int XM, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) pp_gemv_kernel(const GemvArgs a) {
  using L = GemvSmem<MT, XM>;
  constexpr int XB = SplitRows<MT>::kBlock;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int ns = a.nstages;
  GemvShared sh;
  sh.wst = smem;
  sh.xst = smem + L::x_off(ns);
  sh.xs = smem + L::xs_off(ns);
  sh.tile_out = (float*)(smem + L::tile_off(ns, a.kp));
  sh.full = (uint64_t*)(smem + L::bar_off(ns, a.kp));
  sh.empty = sh.full + ns;
  sh.misc = (int32_t*)(smem + L::misc_off(ns, a.kp));
  sh.ns = ns;
  uint8_t* wst = sh.wst;
  uint8_t* xst = sh.xst;
  uint64_t* full = sh.full;
  uint64_t* empty = sh.empty;

  if (a.desc ? bad_step(a.desc, a.capacity, MT) : (a.m_rows < 1 || a.m_rows > MT)) return;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const uint32_t T = (uint32_t)a.tiles * (uint32_t)a.kchunks;
  const uint32_t G = gridDim.x;
  const int i0 = sk_start(blockIdx.x, T, G), i1 = sk_start(blockIdx.x + 1, T, G);

  if (tid == 0) {
    for (int s = 0; s < ns; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
    pdl_launch_dependents();
  }
  __syncthreads();
  // ------------------------------------------------------------------ producer warp
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      const int n_it = i1 - i0;
      const int pre = n_it < ns ? n_it : ns;
      const uint32_t bytes = L::kWBytes + L::kXBytes;
      const int kc = a.kchunks;
      // (tile, chunk) of the next weight block, advanced without divisions.
      int wt = i0 / kc, wc = i0 - (i0 / kc) * kc;
      auto next_w = [&]() {
        const uint16_t* src = a.w + ((size_t)wt * kc + wc) * (kTileRows * kChunkK);
        if (++wc == kc) {
          wc = 0;
          ++wt;
        }
        return src;
      };
      int xc = wc;  // chunk of the next activation block
      auto next_x = [&]() {
        const uint8_t* src = a.xsplit + (size_t)xc * XB;
        if (++xc == kc) xc = 0;
        return src;
      };
      for (int i = 0; i < pre; ++i) {  // weights only: safe before the previous kernel ends
        mbar_arrive_expect_tx(&full[i], bytes);
        bulk_load(wst + (size_t)i * L::kWBytes, next_w(), L::kWBytes, &full[i]);
      }
      pdl_wait();
      if (XM == X_STREAM)
        for (int i = 0; i < pre; ++i) bulk_load(xst + (size_t)i * XB, next_x(), XB, &full[i]);
      int issued = pre;
      int s = pre % ns;
      uint32_t use = pre / ns;
      for (int i = pre; i < n_it; ++i) {
        if (!mbar_wait(&empty[s], (use - 1) & 1)) break;
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_load(wst + (size_t)s * L::kWBytes, next_w(), L::kWBytes, &full[s]);
        if (XM == X_STREAM) bulk_load(xst + (size_t)s * XB, next_x(), XB, &full[s]);
        issued = i + 1;
        if (++s == ns) {
          s = 0;
          ++use;
        }
      }
      if (issued < n_it) {
        gemv_flag(a, ST_TIMEOUT);
        // Let the copies already issued land before the CTA's shared memory goes away.
        for (int j = (issued > ns ? issued - ns : 0); j < issued; ++j)
          mbar_wait(&full[j % ns], (uint32_t)(j / ns) & 1);
      }
    }
    return;
  }


  // ------------------------------------------------------------------ consumer warps
  pdl_wait();
  RingPos rp{0, 0u};
  gemv_consume<MT, XM, EPI>(a, sh, rp, G, blockIdx.x);
}

}  // namespace pp
