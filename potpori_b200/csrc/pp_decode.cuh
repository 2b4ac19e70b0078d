// Single-token step of a whole-model shard as one persistent kernel (the draft model's
// greedy decode and every other 1-row step of a shard that holds all layers).
//
// A 1-row step is a chain of skinny GEMVs and a small attention whose HBM time per layer is
// a few microseconds (Qwen3-0.6B: 31.5 MB of weights and 16 MB of K/V at 2k positions), far
// below the fixed cost of launching, filling and draining six kernels per layer. Here one
// cooperative launch of one CTA per SM runs every layer:
//
//  * Each CTA owns whole output rows of every projection (balanced contiguous ranges of a
//    row-major copy of the weights) and one (KV head, key range) attention unit, so no
//    partial sums cross CTAs and each row is one dot product over the full K.
//  * One producer thread streams the CTA's whole schedule — QKV rows, the unit's cached K/V
//    rows, O rows, gate/up row pairs, down rows, layer after layer — through a ring of 32 KB
//    shared-memory slots with 1-D bulk copies (TMA engine, no multicast). None of it depends
//    on the step's activations, so the ring runs ahead across phase and layer boundaries and
//    the grid barriers overlap with the weight stream.
//  * Eight consumer warps do the phases in order, separated by grid barriers (monotonic
//    arrival counter, release/acquire at GPU scope, bounded by a timer): QKV (input RMSNorm
//    folded in) -> attention (QK-norm, RoPE and the K/V write of the new position by the unit
//    that holds it; the last unit of a KV head to finish merges its splits) -> O + residual
//    -> gate/up with the post-attention norm and SwiGLU -> down + residual. After the last
//    layer the CTAs write the vocabulary head's operand split(x * final_norm) and the
//    per-128-column sums of squares, which the stream-K head kernel consumes.
//
// Arithmetic is the reference's F32 (src/qwen/model.rs:166-183, tiny.rs:20-115): BF16
// weights decoded exactly to F32, F32 products and sums (packed FFMA2), RMSNorm as
// x * (1 / sqrt(mean(x^2) + eps)) * w, attention scores q.k / sqrt(head_dim).
#pragma once
#include "pp_common.cuh"

namespace pp {

constexpr int kDecSlot = 32768;           // bytes per ring slot
constexpr int kDecKvHalf = kDecSlot / 2;  // K rows at 0, V rows at 16 KB of a K/V slot
constexpr uint64_t kDecBarrierNs = 200ull * 1000 * 1000;  // grid barrier time limit

struct DecodeLayer {
  const uint16_t* wqkv;  // [Q + 2 KV][H] row-major BF16 (q rows, k rows, v rows)
  const uint16_t* wo;    // [H][Q]
  const uint16_t* wgu;   // [I][2][H]: gate row j then up row j
  const uint16_t* wd;    // [H][I]
  const float* n_attn;
  const float* n_q;
  const float* n_k;
  const float* n_ffn;
  uint8_t* kc;  // [n_kv][capacity] cache rows (kv_offset layout)
  uint8_t* vc;
};

struct DecodeArgs {
  const DecodeLayer* layers;  // [nl]
  int32_t nl, H, Q, KV, I, hd, nh, nkv, G, V, capacity, embed_kchunks, splits, ss_tiles, nslots;
  int32_t vec_floats;  // floats of the staged-vector region
  float eps, inv_scale;
  const uint16_t* embed;    // tiled embedding table (tiled_offset layout)
  const float* final_norm;  // NULL: no head operand
  const float2* rope;       // [capacity][hd / 2] (cos, sin)
  float* qkv;               // [Q + 2 KV] projections before QK-norm / RoPE
  float* x;                 // [H] residual stream
  float* attn;              // [Q] attention output
  float* act;               // [I] SwiGLU output
  float* part;              // [nh][splits][hd + 4]: max, sum, -, -, unnormalised output
  uint32_t* sync;           // [0] barrier arrivals, [1] abort, [2 + h] finished units of head h
  uint8_t* xw_out;          // split(x * final_norm) (split_offset<1> layout)
  float* ss_out;            // [ss_tiles][kMaxRows] sums of squares of x per 128 columns
  const StepDesc* desc;
  StepResult* res;
};

// Shared memory (from a 1024-aligned base): ring slots | staged vector (xa, xb: float4 units
// of 8 floats split in halves, or the attention scratch) | own residual rows | reduction |
// flags | mbarriers.
struct DecodeSmem {
  int ns, vec_floats, own;
  __host__ __device__ DecodeSmem(int ns_, int vf, int own_) : ns(ns_), vec_floats(vf), own(own_) {}
  __host__ __device__ size_t vec_off() const { return (size_t)ns * kDecSlot; }
  __host__ __device__ size_t own_off() const { return vec_off() + (size_t)vec_floats * 4; }
  __host__ __device__ size_t red_off() const { return own_off() + (((size_t)own * 4 + 15) & ~(size_t)15); }
  __host__ __device__ size_t bar_off() const { return red_off() + 64; }
  __host__ __device__ size_t total() const { return bar_off() + 16 * (size_t)ns + 1024; }
};

// Floats of the staged-vector region: the widest GEMV input (two float4 halves per 8 columns)
// or the attention scratch (queries, new key and value, per-warp partials).
__host__ __device__ inline int decode_vec_floats(int H, int Q, int I, int hd, int G) {
  int k = H > Q ? H : Q;
  k = k > I ? k : I;
  const int att = (G + 2) * hd + kConsumerWarps * G * (hd + 4);
  return k > att ? k : att;
}

// Balanced contiguous share [lo(b), lo(b+1)) of n items over g CTAs.
__device__ __forceinline__ int dec_lo(int n, int b, int g) { return (int)((int64_t)n * b / g); }

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The ring as seen by one side: slot, its phase parity, stages passed.
struct DecRing {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  int ns, slot;
  uint32_t phase, n;
  __device__ __forceinline__ uint8_t* cur() const { return base + (size_t)slot * kDecSlot; }
  __device__ __forceinline__ void advance() {
    ++n;
    if (++slot == ns) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// This CTA's share of every phase; the producer and the consumers derive the same one.
struct DecPlan {
  int q0, q1;     // QKV rows
  int o0, o1;     // O / down rows (one partition of H for both)
  int j0, j1;     // gate/up pairs
  int h, s;       // attention unit (KV head, split); h < 0: none
  int p0, pe;     // cached positions [p0, pe) streamed for the unit
  bool has_new;   // the unit holds the step's own position
  int rps_qkv, rps_o, rps_gu, rps_d, kvps, rowb;
};

__device__ __forceinline__ DecPlan dec_plan(const DecodeArgs& a, int b, int g, int pos) {
  DecPlan p;
  p.q0 = dec_lo(a.Q + 2 * a.KV, b, g);
  p.q1 = dec_lo(a.Q + 2 * a.KV, b + 1, g);
  p.o0 = dec_lo(a.H, b, g);
  p.o1 = dec_lo(a.H, b + 1, g);
  p.j0 = dec_lo(a.I, b, g);
  p.j1 = dec_lo(a.I, b + 1, g);
  const int S = a.splits;
  p.h = -1;
  p.s = 0;
  p.p0 = p.pe = 0;
  p.has_new = false;
  if (b < a.nkv * S) {
    p.h = b / S;
    p.s = b - p.h * S;
    const int c = pos + 1;
    p.p0 = dec_lo(c, p.s, S);
    const int p1 = dec_lo(c, p.s + 1, S);
    p.has_new = p1 == c;  // the last split
    p.pe = p1 < pos ? p1 : pos;
    if (p.pe < p.p0) p.pe = p.p0;
  }
  p.rps_qkv = kDecSlot / (a.H * 2);
  p.rps_o = kDecSlot / (a.Q * 2);
  p.rps_gu = (kDecSlot / (a.H * 2)) & ~1;
  p.rps_d = kDecSlot / (a.I * 2);
  p.rowb = kv_row_bytes(a.hd);
  p.kvps = kDecKvHalf / p.rowb;
  return p;
}

// ---- producer --------------------------------------------------------------------------------
__device__ __forceinline__ bool dec_acquire(DecRing& r) {
  if (r.n < (uint32_t)r.ns) return true;
  // The ring is usually full: poll gently so the consumer warps keep the issue slots.
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(&r.empty[r.slot], r.phase ^ 1u)) return true;
    __nanosleep(128);
  }
  return false;
}

__device__ __forceinline__ bool dec_issue_rows(DecRing& r, const void* src, int rows, int rowbytes,
                                               int rps) {
  const uint8_t* p = (const uint8_t*)src;
  for (int i = 0; i < rows; i += rps) {
    const int n = rows - i < rps ? rows - i : rps;
    if (!dec_acquire(r)) return false;
    const uint32_t bytes = (uint32_t)(n * rowbytes);
    mbar_arrive_expect_tx(&r.full[r.slot], bytes);
    bulk_load(r.cur(), p + (size_t)i * rowbytes, bytes, &r.full[r.slot]);
    r.advance();
  }
  return true;
}

__device__ __forceinline__ bool dec_issue_kv(DecRing& r, const uint8_t* k, const uint8_t* v,
                                             int npos, int rowb, int kvps) {
  for (int i = 0; i < npos; i += kvps) {
    const int n = npos - i < kvps ? npos - i : kvps;
    if (!dec_acquire(r)) return false;
    const uint32_t bytes = (uint32_t)(n * rowb);
    mbar_arrive_expect_tx(&r.full[r.slot], 2 * bytes);
    bulk_load(r.cur(), k + (size_t)i * rowb, bytes, &r.full[r.slot]);
    bulk_load(r.cur() + kDecKvHalf, v + (size_t)i * rowb, bytes, &r.full[r.slot]);
    r.advance();
  }
  return true;
}

// ---- consumers ---------------------------------------------------------------------------------
// Waits for the current slot; false when the copy did not land within the bounded wait.
__device__ __forceinline__ bool dec_take(DecRing& r) { return mbar_wait(&r.full[r.slot], r.phase); }
// Every consumer warp releases every slot once (the empty barrier counts warps).
__device__ __forceinline__ void dec_release(DecRing& r, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(&r.empty[r.slot]);
  r.advance();
}

// Dot products of the `rows` rows of one weight slot (units 16-byte units each) with the
// staged vector; warp w takes the row pairs (2p, 2p + 1), p = w, w + 8, ..., and lane 0 calls
// epi(row, value0, has_second, value1).
template <typename Epi>
__device__ __forceinline__ void dec_dot_slot(const uint8_t* slot, int rows, int units,
                                             const float4* xa, const float4* xb, int warp,
                                             int lane, Epi&& epi) {
  for (int p = warp; 2 * p < rows; p += kConsumerWarps) {
    const int r0 = 2 * p;
    const bool two = r0 + 1 < rows;
    const uint4* w0 = (const uint4*)(slot + (size_t)r0 * units * 16);
    const uint4* w1 = w0 + units;
    float2 a0 = make_float2(0.f, 0.f), a1 = a0, b0 = a0, b1 = a0;
#pragma unroll 4
    for (int u = lane; u < units; u += 32) {
      const float4 x0 = xa[u], x1 = xb[u];
      const uint4 v = w0[u];
      ffma2(a0, make_float2(bf16lo(v.x), bf16hi(v.x)), make_float2(x0.x, x0.y));
      ffma2(a1, make_float2(bf16lo(v.y), bf16hi(v.y)), make_float2(x0.z, x0.w));
      ffma2(a0, make_float2(bf16lo(v.z), bf16hi(v.z)), make_float2(x1.x, x1.y));
      ffma2(a1, make_float2(bf16lo(v.w), bf16hi(v.w)), make_float2(x1.z, x1.w));
      if (two) {
        const uint4 t = w1[u];
        ffma2(b0, make_float2(bf16lo(t.x), bf16hi(t.x)), make_float2(x0.x, x0.y));
        ffma2(b1, make_float2(bf16lo(t.y), bf16hi(t.y)), make_float2(x0.z, x0.w));
        ffma2(b0, make_float2(bf16lo(t.z), bf16hi(t.z)), make_float2(x1.x, x1.y));
        ffma2(b1, make_float2(bf16lo(t.w), bf16hi(t.w)), make_float2(x1.z, x1.w));
      }
    }
    const float s0 = warp_sum((a0.x + a0.y) + (a1.x + a1.y));
    const float s1 = two ? warp_sum((b0.x + b0.y) + (b1.x + b1.y)) : 0.f;
    if (lane == 0) epi(r0, s0, two, s1);
  }
}

// Consumes one weight segment of `rows` rows; `live` false only releases the slots.
template <typename Epi>
__device__ __forceinline__ bool dec_rows(DecRing& r, bool live, int rows, int rowbytes, int rps,
                                         const float4* xa, const float4* xb, int warp, int lane,
                                         Epi&& epi) {
  for (int i = 0; i < rows; i += rps) {
    const int n = rows - i < rps ? rows - i : rps;
    if (!dec_take(r)) return false;
    if (live)
      dec_dot_slot(r.cur(), n, rowbytes >> 4, xa, xb, warp, lane,
                   [&](int rr, float s0, bool two, float s1) { epi(i + rr, s0, two, s1); });
    dec_release(r, lane);
  }
  return true;
}

// Stages K floats of src (times w when given) into the unit-split vector; returns the sum of
// squares of src, reduced in the same order in every CTA.
__device__ __forceinline__ float dec_stage_vec(const float* src, const float* w, int K, float4* xa,
                                               float4* xb, float* red, int tid) {
  constexpr int T = kConsumerWarps * 32, B = 4;  // float4s per thread per batch of loads
  float ss = 0.f;
  for (int q0 = 0; q0 < (K >> 2); q0 += B * T) {
    float4 v[B], ww[B];
#pragma unroll
    for (int k = 0; k < B; ++k) {  // every load of the batch in flight together
      const int q = q0 + tid + k * T;
      const bool in = q < (K >> 2);
      v[k] = in ? __ldcg((const float4*)src + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      ww[k] = (in && w) ? ((const float4*)w)[q] : make_float4(1.f, 1.f, 1.f, 1.f);
    }
#pragma unroll
    for (int k = 0; k < B; ++k) {
      const int q = q0 + tid + k * T;
      if (q < (K >> 2)) {
        float4 x = v[k];
        ss += (x.x * x.x + x.y * x.y) + (x.z * x.z + x.w * x.w);
        if (w) {
          x.x *= ww[k].x;
          x.y *= ww[k].y;
          x.z *= ww[k].z;
          x.w *= ww[k].w;
        }
        ((q & 1) ? xb : xa)[q >> 1] = x;
      }
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  consumer_sync();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) t += red[i];
  consumer_sync();  // red is free again
  return t;
}

// Grid barrier among the consumers of all CTAs (the producers never wait on it): barrier
// number k completes when the arrival counter reaches k * gridDim.x. False when the step
// was aborted (a barrier of some CTA ran out of time).
__device__ __forceinline__ bool dec_grid_sync(const DecodeArgs& a, uint32_t target, int* flag,
                                              int tid) {
  consumer_sync();
  if (tid == 0) {
    int ok = 1;
    red_release_gpu(&a.sync[0], 1);
    const uint64_t t0 = global_timer_ns();
    for (uint32_t n = 1; ld_acquire_gpu(&a.sync[0]) < target; ++n) {
      if ((n & 63) == 0) {
        if (ld_acquire_gpu(&a.sync[1])) {
          ok = 0;
          break;
        }
        if (global_timer_ns() - t0 > kDecBarrierNs) {
          atomicOr(&a.res->status, ST_TIMEOUT);
          atomicExch(&a.sync[1], 1u);
          ok = 0;
          break;
        }
      }
    }
    *flag = ok;
  }
  consumer_sync();
  return *flag != 0;
}

// Attention unit (KV head h, split s) for the single query position pos: QK-RMSNorm + RoPE
// of the G query heads and of the new key (tiny.rs:24-37), the new K/V row written by the
// unit that holds pos, online softmax over the streamed cached rows (tiny.rs:77-101), the
// unit's partial (max, sum, output) per query head, and the merge of the head's splits by
// the last unit to finish.
template <int G>  // query heads per KV head (a.G)
__device__ __forceinline__ bool dec_attention(const DecodeArgs& a, const DecodeLayer& L,
                                              const DecPlan& P, DecRing& r, bool live, int pos,
                                              int layer, float* vec, int* flag, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int hd = a.hd, half = hd >> 1, h = P.h;
  float* qs = vec;             // [G][hd]
  float* kn = qs + G * hd;     // [hd]
  float* vn = kn + hd;         // [hd]
  float* mrg = vn + hd;        // [warps][G][hd + 4]
  if (live) {
    // The new value row rides along with the first batch of loads (hd <= 256 threads).
    const float vnew = (P.has_new && tid < hd) ? __ldcg(a.qkv + a.Q + a.KV + h * hd + tid) : 0.f;
    for (int p = warp; p <= G; p += kConsumerWarps) {
      const bool isq = p < G;
      if (!isq && !P.has_new) continue;
      const float* src = a.qkv + (isq ? (h * G + p) * hd : a.Q + h * hd);
      const float* w = isq ? L.n_q : L.n_k;
      const float2* rp = a.rope + (size_t)pos * half;
      // One batch of loads per lane: its raw values, norm weights and (cos, sin) pairs for
      // dims i and i + half, i = lane + 32 t (head_dim <= 128).
      float x0[2], x1[2], w0[2], w1[2];
      float2 cs[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int i = lane + 32 * t;
        const bool in = i < half;
        x0[t] = in ? __ldcg(src + i) : 0.f;
        x1[t] = in ? __ldcg(src + i + half) : 0.f;
        w0[t] = in ? w[i] : 0.f;
        w1[t] = in ? w[i + half] : 0.f;
        cs[t] = in ? rp[i] : make_float2(0.f, 0.f);
      }
      const float ssq = warp_sum((x0[0] * x0[0] + x1[0] * x1[0]) + (x0[1] * x0[1] + x1[1] * x1[1]));
      const float rms = sqrtf(ssq / (float)hd + a.eps);
      float* dst = isq ? qs + p * hd : kn;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int i = lane + 32 * t;
        if (i < half) {
          const float y0 = x0[t] / rms * w0[t], y1 = x1[t] / rms * w1[t];
          dst[i] = y0 * cs[t].x - y1 * cs[t].y;
          dst[i + half] = y1 * cs[t].x + y0 * cs[t].y;
        }
      }
    }
    if (P.has_new && tid < hd) vn[tid] = vnew;
    consumer_sync();
    if (P.has_new) {
      const size_t off = ((size_t)h * a.capacity + pos) * kv_row_bytes(hd);
      for (int i = tid; i < hd; i += kConsumerWarps * 32) {
        kv_store(L.kc + off, pos, i, hd, kn[i]);
        kv_store(L.vc + off, pos, i, hd, vn[i]);
      }
    }
  }
  // Lane l holds dims 4l..4l+3 of every query head and of the running outputs.
  const bool act = 4 * lane < hd;
  const int d0 = 4 * lane;
  float q[G][4], o[G][4], m[G], l[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[g][j] = 0.f;
      q[g][j] = (live && act) ? qs[g * hd + d0 + j] : 0.f;
    }
  }
  // Online softmax over one or two keys (B valid when vb): the dot products of both keys are
  // reduced together so their shuffle chains overlap, then the state takes A, then B.
  auto visit2 = [&](const float (&ka)[4], const float (&va)[4], bool vb, const float (&kb)[4],
                    const float (&vb4)[4]) {
    float sa[G], sb[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sa[g] = (q[g][0] * ka[0] + q[g][1] * ka[1]) + (q[g][2] * ka[2] + q[g][3] * ka[3]);
      sb[g] = (q[g][0] * kb[0] + q[g][1] * kb[1]) + (q[g][2] * kb[2] + q[g][3] * kb[3]);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        sa[g] += __shfl_xor_sync(0xffffffffu, sa[g], off);
        sb[g] += __shfl_xor_sync(0xffffffffu, sb[g], off);
      }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float sc = sa[g] * a.inv_scale;
      float mn = fmaxf(m[g], sc);
      float al = __expf(m[g] - mn);  // 0 for the first key (m = -inf)
      float pr = __expf(sc - mn);
      l[g] = l[g] * al + pr;
#pragma unroll
      for (int j = 0; j < 4; ++j) o[g][j] = o[g][j] * al + pr * va[j];
      m[g] = mn;
      if (vb) {
        sc = sb[g] * a.inv_scale;
        mn = fmaxf(m[g], sc);
        al = __expf(m[g] - mn);
        pr = __expf(sc - mn);
        l[g] = l[g] * al + pr;
#pragma unroll
        for (int j = 0; j < 4; ++j) o[g][j] = o[g][j] * al + pr * vb4[j];
        m[g] = mn;
      }
    }
  };
  auto load_kv = [&](const uint8_t* ks, const uint8_t* vs, int i, int j, float (&k)[4],
                     float (&v)[4]) {
    const uint8_t* kr = ks + (size_t)i * P.rowb;
    const uint8_t* vr = vs + (size_t)i * P.rowb;
    const uint2 kh = *(const uint2*)(kr + kv_offset(j, d0, 0, hd));
    const uint2 kl = *(const uint2*)(kr + kv_offset(j, d0, 1, hd));
    const uint2 vh = *(const uint2*)(vr + kv_offset(j, d0, 0, hd));
    const uint2 vl = *(const uint2*)(vr + kv_offset(j, d0, 1, hd));
    k[0] = bf16lo(kh.x) + bf16lo(kl.x);
    k[1] = bf16hi(kh.x) + bf16hi(kl.x);
    k[2] = bf16lo(kh.y) + bf16lo(kl.y);
    k[3] = bf16hi(kh.y) + bf16hi(kl.y);
    v[0] = bf16lo(vh.x) + bf16lo(vl.x);
    v[1] = bf16hi(vh.x) + bf16hi(vl.x);
    v[2] = bf16lo(vh.y) + bf16lo(vl.y);
    v[3] = bf16hi(vh.y) + bf16hi(vl.y);
  };
  const int npos = P.pe - P.p0;
  for (int i0 = 0; i0 < npos; i0 += P.kvps) {
    const int n = npos - i0 < P.kvps ? npos - i0 : P.kvps;
    if (!dec_take(r)) return false;
    if (live) {
      const uint8_t* ks = r.cur();
      const uint8_t* vs = ks + kDecKvHalf;
      for (int i = warp; i < n; i += 2 * kConsumerWarps) {
        const int ib = i + kConsumerWarps;
        const bool vb = ib < n;
        float ka[4] = {0.f, 0.f, 0.f, 0.f}, va[4] = {0.f, 0.f, 0.f, 0.f};
        float kb[4] = {0.f, 0.f, 0.f, 0.f}, vbv[4] = {0.f, 0.f, 0.f, 0.f};
        if (act) {
          load_kv(ks, vs, i, P.p0 + i0 + i, ka, va);
          if (vb) load_kv(ks, vs, ib, P.p0 + i0 + ib, kb, vbv);
        }
        visit2(ka, va, vb, kb, vbv);
      }
    }
    dec_release(r, lane);
  }
  if (!live) return true;
  if (P.has_new && warp == (npos % kConsumerWarps)) {
    float k[4] = {0.f, 0.f, 0.f, 0.f}, v[4] = {0.f, 0.f, 0.f, 0.f};
    if (act)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        k[j] = kn[d0 + j];
        v[j] = vn[d0 + j];
      }
    visit2(k, v, false, k, v);
  }
  // Merge the warps' partials: thread t handles (head g, dim d) of the unit's record.
  const int stride = hd + 4;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float* mw = mrg + (size_t)(warp * G + g) * stride;
    if (lane == 0) {
      mw[0] = m[g];
      mw[1] = l[g];
    }
    if (act)
#pragma unroll
      for (int j = 0; j < 4; ++j) mw[4 + d0 + j] = o[g][j];
  }
  consumer_sync();
  const int S = a.splits;
  for (int e = tid; e < G * hd; e += kConsumerWarps * 32) {
    const int g = e / hd, d = e - g * hd;
    float M = -INFINITY;
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mrg[(size_t)(w * G + g) * stride]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY)
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float* mw = mrg + (size_t)(w * G + g) * stride;
        const float f = mw[0] == -INFINITY ? 0.f : __expf(mw[0] - M);
        Ls += mw[1] * f;
        O += mw[4 + d] * f;
      }
    float* rec = a.part + ((size_t)(h * G + g) * S + P.s) * stride;
    if (d == 0) {
      rec[0] = M;
      rec[1] = Ls;
    }
    rec[4 + d] = O;
  }
  consumer_sync();
  // The head's counter counts the units of every layer so far: the last of this layer's S.
  if (tid == 0)
    *flag = atom_add_acq_rel_gpu(&a.sync[2 + h], 1u) == (uint32_t)((layer + 1) * S - 1);
  consumer_sync();
  if (*flag) {
    // Last unit of head h: merge the S splits (exp(max_s - max) weights, split order). The
    // splits' maxima and sums come in one batch of loads, then each thread's S outputs.
    float* Ms = mrg;           // [G][S] (the warps' partials are no longer needed)
    float* Ss = mrg + G * S;   // [G][S]
    for (int e = tid; e < G * S; e += kConsumerWarps * 32) {
      const int g = e / S, sp = e - g * S;
      const float2 ml = __ldcg((const float2*)(a.part + ((size_t)(h * G + g) * S + sp) * stride));
      Ms[e] = ml.x;
      Ss[e] = ml.y;
    }
    consumer_sync();
    for (int e = tid; e < G * hd; e += kConsumerWarps * 32) {
      const int g = e / hd, d = e - g * hd;
      const float* col = a.part + (size_t)(h * G + g) * S * stride + 4 + d;
      float pv[32];
#pragma unroll
      for (int sp = 0; sp < 32; ++sp) pv[sp] = sp < S ? __ldcg(col + (size_t)sp * stride) : 0.f;
      float M = -INFINITY;
      for (int sp = 0; sp < S; ++sp) M = fmaxf(M, Ms[g * S + sp]);
      float Ls = 0.f, O = 0.f;
#pragma unroll
      for (int sp = 0; sp < 32; ++sp) {
        if (sp < S) {
          const float ms = Ms[g * S + sp];
          const float f = ms == -INFINITY ? 0.f : expf(ms - M);
          Ls += Ss[g * S + sp] * f;
          O += pv[sp] * f;
        }
      }
      for (int sp = 32; sp < S; ++sp) {
        const float ms = Ms[g * S + sp];
        const float f = ms == -INFINITY ? 0.f : expf(ms - M);
        Ls += Ss[g * S + sp] * f;
        O += __ldcg(col + (size_t)sp * stride) * f;
      }
      a.attn[(h * G + g) * hd + d] = O / Ls;
    }
  }
  return true;
}

template <int G>  // query heads per KV head (a.G)
__global__ void __launch_bounds__(kGemvThreads, 1) pp_decode_step_kernel(const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int NG = gridDim.x, b = blockIdx.x, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int own_cap = (a.H + NG - 1) / NG + 1;
  const DecodeSmem lay(a.nslots, a.vec_floats, own_cap);
  DecRing r;
  r.base = smem;
  r.full = (uint64_t*)(smem + lay.bar_off());
  r.empty = r.full + a.nslots;
  r.ns = a.nslots;
  r.slot = 0;
  r.phase = 0;
  r.n = 0;
  float* vec = (float*)(smem + lay.vec_off());
  float4* xa = (float4*)vec;
  float4* xb = xa + (a.vec_floats >> 3);
  float* xown = (float*)(smem + lay.own_off());
  float* red = (float*)(smem + lay.red_off());
  int* flag = (int*)(red + kConsumerWarps);

  if (bad_step(a.desc, a.capacity, 1)) return;
  const int pos = a.desc->pos, tok = a.desc->tokens[0];
  if (tok < 0 || tok >= a.V) return;  // pp_step_begin_kernel reports it
  if (tid == 0) {
    for (int i = 0; i < a.nslots; ++i) {
      mbar_init(&r.full[i], 1);
      mbar_init(&r.empty[i], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  const DecPlan P = dec_plan(a, b, NG, pos);

  // ------------------------------------------------------------------ producer thread
  if (warp == kConsumerWarps) {
    if (lane != 0) return;
    bool ok = true;
    for (int l = 0; l < a.nl && ok; ++l) {
      const DecodeLayer& L = a.layers[l];
      ok = dec_issue_rows(r, L.wqkv + (size_t)P.q0 * a.H, P.q1 - P.q0, a.H * 2, P.rps_qkv);
      if (ok && P.h >= 0) {
        const size_t off = ((size_t)P.h * a.capacity + P.p0) * P.rowb;
        ok = dec_issue_kv(r, L.kc + off, L.vc + off, P.pe - P.p0, P.rowb, P.kvps);
      }
      ok = ok && dec_issue_rows(r, L.wo + (size_t)P.o0 * a.Q, P.o1 - P.o0, a.Q * 2, P.rps_o);
      ok = ok && dec_issue_rows(r, L.wgu + (size_t)2 * P.j0 * a.H, 2 * (P.j1 - P.j0), a.H * 2, P.rps_gu);
      ok = ok && dec_issue_rows(r, L.wd + (size_t)P.o0 * a.I, P.o1 - P.o0, a.I * 2, P.rps_d);
    }
    if (!ok) {
      atomicOr(&a.res->status, ST_TIMEOUT);
      atomicExch(&a.sync[1], 1u);
      // Let the copies already issued land before the CTA's shared memory goes away.
      const uint32_t first = r.n > (uint32_t)r.ns ? r.n - r.ns : 0;
      for (uint32_t j = first; j < r.n; ++j)
        mbar_wait(&r.full[j % r.ns], (j / r.ns) & 1u);
    }
    return;
  }

  // ------------------------------------------------------------------ consumer warps
  bool live = true, lost = false;  // lost: a ring slot never landed
  uint32_t nb = 0;
  for (int l = 0; l < a.nl && !lost; ++l) {
    const DecodeLayer& L = a.layers[l];
    // QKV with the input RMSNorm; layer 0 gathers the token's embedding row
    // (src/qwen/model.rs:239-241).
    float rinv = 0.f;
    if (live) {
      float ss;
      if (l == 0) {
        float t = 0.f;
        for (int q = tid; q < (a.H >> 2); q += kConsumerWarps * 32) {
          float4 v;
          v.x = __uint_as_float((uint32_t)a.embed[tiled_offset(tok, 4 * q + 0, a.embed_kchunks)] << 16);
          v.y = __uint_as_float((uint32_t)a.embed[tiled_offset(tok, 4 * q + 1, a.embed_kchunks)] << 16);
          v.z = __uint_as_float((uint32_t)a.embed[tiled_offset(tok, 4 * q + 2, a.embed_kchunks)] << 16);
          v.w = __uint_as_float((uint32_t)a.embed[tiled_offset(tok, 4 * q + 3, a.embed_kchunks)] << 16);
          const int n0 = 4 * q;
          if (n0 + 3 >= P.o0 && n0 < P.o1) {
            if (n0 + 0 >= P.o0 && n0 + 0 < P.o1) xown[n0 + 0 - P.o0] = v.x;
            if (n0 + 1 >= P.o0 && n0 + 1 < P.o1) xown[n0 + 1 - P.o0] = v.y;
            if (n0 + 2 >= P.o0 && n0 + 2 < P.o1) xown[n0 + 2 - P.o0] = v.z;
            if (n0 + 3 >= P.o0 && n0 + 3 < P.o1) xown[n0 + 3 - P.o0] = v.w;
          }
          t += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
          const float4 ww = ((const float4*)L.n_attn)[q];
          v.x *= ww.x;
          v.y *= ww.y;
          v.z *= ww.z;
          v.w *= ww.w;
          ((q & 1) ? xb : xa)[q >> 1] = v;
        }
        t = warp_sum(t);
        if (lane == 0) red[warp] = t;
        consumer_sync();
        ss = 0.f;
#pragma unroll
        for (int i = 0; i < kConsumerWarps; ++i) ss += red[i];
        consumer_sync();
      } else {
        ss = dec_stage_vec(a.x, L.n_attn, a.H, xa, xb, red, tid);
      }
      rinv = 1.0f / sqrtf(ss / (float)a.H + a.eps);
    }
    if (!dec_rows(r, live, P.q1 - P.q0, a.H * 2, P.rps_qkv, xa, xb, warp, lane,
                  [&](int rr, float s0, bool two, float s1) {
                    a.qkv[P.q0 + rr] = s0 * rinv;
                    if (two) a.qkv[P.q0 + rr + 1] = s1 * rinv;
                  })) {
      lost = true;
      break;
    }
    live = live && dec_grid_sync(a, ++nb * (uint32_t)NG, flag, tid);
    // Attention.
    if (P.h >= 0 && !dec_attention<G>(a, L, P, r, live, pos, l, vec, flag, tid)) {
      lost = true;
      break;
    }
    live = live && dec_grid_sync(a, ++nb * (uint32_t)NG, flag, tid);
    // O projection + residual (src/qwen/model.rs:304-306).
    if (live) dec_stage_vec(a.attn, nullptr, a.Q, xa, xb, red, tid);
    if (!dec_rows(r, live, P.o1 - P.o0, a.Q * 2, P.rps_o, xa, xb, warp, lane,
                  [&](int rr, float s0, bool two, float s1) {
                    float v = xown[rr] + s0;
                    xown[rr] = v;
                    a.x[P.o0 + rr] = v;
                    if (two) {
                      v = xown[rr + 1] + s1;
                      xown[rr + 1] = v;
                      a.x[P.o0 + rr + 1] = v;
                    }
                  })) {
      lost = true;
      break;
    }
    live = live && dec_grid_sync(a, ++nb * (uint32_t)NG, flag, tid);
    // gate/up with the post-attention RMSNorm, SwiGLU (tiny.rs:111-115).
    if (live) {
      const float ss = dec_stage_vec(a.x, L.n_ffn, a.H, xa, xb, red, tid);
      rinv = 1.0f / sqrtf(ss / (float)a.H + a.eps);
    }
    if (!dec_rows(r, live, 2 * (P.j1 - P.j0), a.H * 2, P.rps_gu, xa, xb, warp, lane,
                  [&](int rr, float s0, bool, float s1) {
                    const float g = s0 * rinv, u = s1 * rinv;
                    a.act[P.j0 + (rr >> 1)] = g / (1.0f + expf(-g)) * u;
                  })) {
      lost = true;
      break;
    }
    live = live && dec_grid_sync(a, ++nb * (uint32_t)NG, flag, tid);
    // down + residual.
    if (live) dec_stage_vec(a.act, nullptr, a.I, xa, xb, red, tid);
    if (!dec_rows(r, live, P.o1 - P.o0, a.I * 2, P.rps_d, xa, xb, warp, lane,
                  [&](int rr, float s0, bool two, float s1) {
                    float v = xown[rr] + s0;
                    xown[rr] = v;
                    a.x[P.o0 + rr] = v;
                    if (two) {
                      v = xown[rr + 1] + s1;
                      xown[rr + 1] = v;
                      a.x[P.o0 + rr + 1] = v;
                    }
                  })) {
      lost = true;
      break;
    }
    live = live && dec_grid_sync(a, ++nb * (uint32_t)NG, flag, tid);
  }
  if (lost) {
    if (tid == 0) {
      atomicOr(&a.res->status, ST_TIMEOUT);
      atomicExch(&a.sync[1], 1u);
    }
    return;
  }
  if (!live || !a.final_norm) return;
  // The vocabulary head's operand: split(x * final_norm) and the sums of squares of x per
  // 128 columns (the layout pp_input_prep_kernel writes).
  for (int t = b; t < a.ss_tiles; t += NG) {
    float v = 0.f;
    const int n = t * 128 + tid;
    if (tid < 128 && n < a.H) {
      v = __ldcg(a.x + n);
      store_split<1>(a.xw_out, 0, n, v * a.final_norm[n]);
    }
    const float sq = warp_sum(v * v);
    if (lane == 0) red[warp] = sq;
    consumer_sync();
    if (tid == 0) a.ss_out[t * kMaxRows] = (red[0] + red[1]) + (red[2] + red[3]);
    consumer_sync();
  }
}

// Row-major copies of the packed weights for the decode kernel: dst[r][c] = W[row(r)][c]
// with row(r) = r (QKV, O, down) or, for the gate/up pairs (mode 1), gate row r/2 or up row
// r/2 of the 64-row interleaved blocks.
__global__ void pp_untile_rows_kernel(uint16_t* dst, const uint16_t* src, int64_t rows, int64_t cols,
                                   int64_t kchunks, int32_t mode) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    int64_t pr = r;
    if (mode == 1) {
      const int64_t j = r >> 1;
      pr = (j / (kTileRows / 2)) * kTileRows + (j % (kTileRows / 2)) + (r & 1) * (kTileRows / 2);
    }
    dst[i] = src[tiled_offset(pr, c, kchunks)];
  }
}

}  // namespace pp
