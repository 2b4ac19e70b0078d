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
//  * In a GEMV slot the K dimension is split over the eight warps: a lane holds its slice of
//    the input vector in registers for the whole phase and reads each weight byte once from
//    shared memory (the weight rows are stored with a per-row swizzle of their 16-byte units,
//    so the lanes of a warp hit distinct bank groups); the warps' partial sums meet in a small
//    double-buffered table.
//  * In the attention a key is eight lanes (16 head dims each): a warp walks four keys at a
//    time, each lane group with its own running max, sum and output, merged at the end.
//
// Arithmetic is the reference's F32 (src/qwen/model.rs:166-183, tiny.rs:20-115): BF16
// weights decoded exactly to F32, F32 products and sums (packed FFMA2), RMSNorm as
// x * (1 / sqrt(mean(x^2) + eps)) * w, attention scores q.k / sqrt(head_dim).
#pragma once
#include "pp_common.cuh"
#include "pp_gemv.cuh"  // ldmatrix_x4, mma_bf16

namespace pp {

constexpr int kDecSlot = 32768;           // bytes per ring slot
constexpr int kDecKvHalf = kDecSlot / 2;  // K rows at 0, V rows at 16 KB of a K/V slot
constexpr uint64_t kDecBarrierNs = 200ull * 1000 * 1000;  // default barrier time limit
constexpr int kDecKAlign = 512;           // K of the weight copies: a multiple of 8 warps x 64
constexpr int kDecHd = 128;               // head size the attention takes
// Three warpgroups: two of consumer warps and one whose first thread is the producer. The block
// launches at 168 registers a thread (65,536 / 384); the producer warpgroup gives back all but
// 40 and the consumer warpgroups take them: 128 x 40 + 256 x 232 = 384 x 168.
constexpr int kDecThreads = 384;
constexpr int kDecMaxAdds = 8;  // KV heads whose O shares the gate/up staging sums
constexpr int kDecProducerRegs = 40, kDecConsumerRegs = 232;
static_assert(128 * kDecProducerRegs + 256 * kDecConsumerRegs <= kDecThreads * 168,
              "the register split must fit the launch's registers");

// K of a decode weight copy (zero columns past K): a multiple of 512, and of 1024 above 4096
// and 2048 above 8192, so the kp / 64 units of a warp's columns split evenly over the lanes of
// a row (32 / dec_slot_rows(kp) lanes).
__host__ __device__ inline int dec_kpad(int k) {
  const int a = k > 8192 ? 2048 : k > 4096 ? 1024 : kDecKAlign;
  return (k + a - 1) / a * a;
}
// Rows per weight slot for rows of kp columns: the largest power of two <= 32 that fits (a lane
// per row at 32, so at most 32).
__host__ __device__ inline int dec_slot_rows(int kp) {
  int r = 32;
  while (r > 1 && r * kp * 2 > kDecSlot) r >>= 1;
  return r;
}
// Element offset of (row r, column c) in a decode weight copy of kp columns per row: the
// 16-byte unit c / 8 of row r sits at (c / 8) ^ (r & 7), inside its 128-byte group, so the
// lanes reading one unit of eight consecutive rows hit eight different bank groups.
__host__ __device__ inline int64_t dec_w_offset(int64_t r, int64_t c, int64_t kp) {
  return r * kp + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7);
}

struct DecodeLayer {
  const uint16_t* wqkv;  // [Q + 2 KV][kH] (q rows, k rows, v rows), dec_w_offset layout
  const uint16_t* wo;    // [n_kv][H][kO]: per KV head, its G query heads' columns of O
  const uint16_t* wgu;   // [I][2][kH]: gate row j then up row j
  const uint16_t* wd;    // [H][kI]
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
  int32_t kH, kQ, kI;  // K of the weight copies (dec_kpad of H, Q, I)
  int32_t kO;          // K of the per-head O copy: G * head_dim
  int32_t vec_floats;  // floats of the staged-vector region
  int32_t extra_arrivals;  // added to every grid barrier's target (a test of the time limit)
  uint64_t wait_ns;        // time limit of the grid and head barriers
  float eps, inv_scale;
  const uint16_t* embed;    // tiled embedding table (tiled_offset layout)
  const float* final_norm;  // NULL: no head operand
  const float2* rope;       // [capacity][hd / 2] (cos, sin)
  float* qkv;               // [Q + 2 KV] projections before QK-norm / RoPE
  float* x;                 // [H] residual stream
  float* attn;              // [Q] attention output (unused: each head's stays on chip)
  float* opart;             // [n_kv][H] O projection of each KV head's query heads
  float* act;               // [I] SwiGLU output
  float* part;              // [nh][splits][hd + 4]: max, sum, -, -, unnormalised output
  uint32_t* sync;           // [0] barrier arrivals, [1] abort, [2 + h] units of head h done
  uint8_t* xw_out;          // split(x * final_norm) (split_offset<1> layout)
  float* ss_out;            // [ss_tiles][kMaxRows] sums of squares of x per 128 columns
  const StepDesc* desc;
  StepResult* res;
};

// Shared memory (from a 1024-aligned base): ring slots | staged vector (the phase's input,
// padded, or the attention scratch) | own residual rows | warp partials [rows][8] |
// reduction | flags | mbarriers.
struct DecodeSmem {
  int ns, vec_floats, own, prow;
  __host__ __device__ DecodeSmem(int ns_, int vf, int own_, int prow_)
      : ns(ns_), vec_floats(vf), own(own_), prow(prow_) {}
  __host__ __device__ size_t vec_off() const { return (size_t)ns * kDecSlot; }
  __host__ __device__ size_t own_off() const { return vec_off() + (size_t)vec_floats * 4; }
  __host__ __device__ size_t part_off() const { return own_off() + (((size_t)own * 4 + 15) & ~(size_t)15); }
  __host__ __device__ size_t red_off() const { return part_off() + (size_t)prow * kConsumerWarps * 4; }
  __host__ __device__ size_t bar_off() const { return red_off() + 64; }
  __host__ __device__ size_t total() const { return bar_off() + 16 * (size_t)ns + 1024; }
};

// Floats of the staged-vector region: the widest padded GEMV input (a pad of 4 floats per
// slice, a slice at least 4 units) or the attention scratch (queries, new key and value,
// per-warp partials; the merge of a head's splits reuses it).
__host__ __device__ inline int decode_att_floats(int hd, int G) {
  return (G + 2) * hd + kConsumerWarps * G * (hd + 4);
}
__host__ __device__ inline int decode_vec_floats(int H, int Q, int I, int hd, int G) {
  int k = dec_kpad(H) > dec_kpad(Q) ? dec_kpad(H) : dec_kpad(Q);
  k = k > dec_kpad(I) ? k : dec_kpad(I);
  k += k / 8;
  // The attention scratch, then the head's merged output for its O rows (padded, at least one
  // unit per slice: 4 floats of pad per 8).
  const int att = decode_att_floats(hd, G) + G * hd * 3 / 2 + 16;
  return k > att ? k : att;
}

// Balanced contiguous share [lo(b), lo(b+1)) of n items over g CTAs.
__device__ __forceinline__ int dec_lo(int n, int b, int g) { return (int)((int64_t)n * b / g); }

// Rows of the partial table: the most rows of one GEMV phase a CTA of a g-CTA grid gets
// (QKV rows, gate/up rows, down rows, or an attention unit's rows of its head's O block).
__host__ __device__ inline int decode_part_rows(int H, int Q, int KV, int I, int nkv, int g) {
  const int S = g / nkv > 0 ? g / nkv : 1;
  const int a = (Q + 2 * KV + g - 1) / g, b = (2 * I + 2 * g - 1) / g, c = (H + g - 1) / g;
  const int o = (H + S - 1) / S;
  int m = a > b ? a : b;
  m = m > c ? m : c;
  return (m > o ? m : o) + 2;
}

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
  int r0, r1;     // the unit's rows of its head's O block
  int rps_qkv, rps_oh, rps_gu, rps_d, kvps, rowb;
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
  p.r0 = p.r1 = 0;
  if (b < a.nkv * S) {
    p.h = b / S;
    p.s = b - p.h * S;
    p.r0 = dec_lo(a.H, p.s, S);
    p.r1 = dec_lo(a.H, p.s + 1, S);
    const int c = pos + 1;
    p.p0 = dec_lo(c, p.s, S);
    const int p1 = dec_lo(c, p.s + 1, S);
    p.has_new = p1 == c;  // the last split
    p.pe = p1 < pos ? p1 : pos;
    if (p.pe < p.p0) p.pe = p.p0;
  }
  p.rps_qkv = dec_slot_rows(a.kH);
  p.rps_oh = dec_slot_rows(a.kO);
  p.rps_gu = dec_slot_rows(a.kH);  // an even number: gate/up pairs never straddle two slots
  p.rps_d = dec_slot_rows(a.kI);
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

// A lane's part of one GEMV phase: slots of R rows of kp columns; the lanes of a warp take the
// rows (lpr = 32 / R lanes per row), and warp w the columns [w kp / 8, (w + 1) kp / 8), of
// which the lane takes upl 16-byte units: unit u0 + us t of the whole row for t < upl.
// The eight lanes of a quarter warp (one shared-memory wavefront of 16-byte loads) must read
// eight different bank groups:
//  * R >= 8: lane l takes row l % R and the contiguous slice l / R of the warp's units; a
//    quarter warp is eight consecutive rows of one slice, whose row swizzles differ;
//  * R < 8 (lpr >= 8): lane l takes row l / lpr and every lpr-th unit from l % lpr; a quarter
//    warp is eight consecutive units of one row.
struct DecLane {
  int lpr, upl, row, sub, u0, us;
};

__device__ __forceinline__ DecLane dec_lane(int kp, int R, int warp, int lane) {
  DecLane d;
  d.lpr = 32 / R;
  d.upl = (kp >> 6) / d.lpr;
  if (R >= 8) {
    d.row = lane & (R - 1);
    d.sub = lane / R;
    d.u0 = warp * (kp >> 6) + d.sub * d.upl;
    d.us = 1;
  } else {
    d.row = lane / d.lpr;
    d.sub = lane - d.row * d.lpr;
    d.u0 = warp * (kp >> 6) + d.sub;
    d.us = d.lpr;
  }
  return d;
}

// The lane's units of the staged input vector, 8 floats per unit, held for the whole phase.
__device__ __forceinline__ void dec_load_x(const float* vec, const DecLane& d, float4 (&x)[16]) {
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const bool in = t < d.upl;
    const float4* v4 = (const float4*)(vec + 8 * (d.u0 + d.us * t));
    x[2 * t] = in ? v4[0] : make_float4(0.f, 0.f, 0.f, 0.f);
    x[2 * t + 1] = in ? v4[1] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Stages K floats of src plus, when given, the `nadd` vectors add[j][0..K) (the heads' shares
// of O, summed in head order), times w when given, into vec[0..kp) (zeros past K); the CTA's
// own rows [o0, o1) of the sum also go to xown when given. Returns the sum of squares of the
// sum, reduced in the same order in every CTA.
__device__ __forceinline__ float dec_stage_vec(const float* src, const float* add, int nadd,
                                               const float* w, int K, int kp, float* vec,
                                               float* red, int tid, float* xown, int o0, int o1) {
  constexpr int T = kConsumerWarps * 32, B = 4;  // float4s per thread per batch of loads
  const int step = add ? 1 : B;                   // with adds: one float4 of every source
  float ss = 0.f;
  for (int q0 = 0; q0 < (kp >> 2); q0 += step * T) {
    float4 v[B], ww[B];
    if (add) {
      // Every source's float4 in flight together, summed in head order.
      const int q = q0 + tid;
      const bool in = q < (K >> 2);
      float4 t[kDecMaxAdds];
#pragma unroll
      for (int j = 0; j < kDecMaxAdds; ++j)
        if (j < nadd)
          t[j] = in ? __ldcg((const float4*)(add + (size_t)j * K) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[0] = in ? __ldcg((const float4*)src + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      ww[0] = (in && w) ? ((const float4*)w)[q] : make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
      for (int j = 0; j < kDecMaxAdds; ++j) {
        if (j < nadd) {
          v[0].x += t[j].x;
          v[0].y += t[j].y;
          v[0].z += t[j].z;
          v[0].w += t[j].w;
        }
      }
#pragma unroll
      for (int k = 1; k < B; ++k) v[k] = ww[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
#pragma unroll
      for (int k = 0; k < B; ++k) {  // every load of the batch in flight together
        const int q = q0 + tid + k * T;
        const bool in = q < (K >> 2);
        v[k] = in ? __ldcg((const float4*)src + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        ww[k] = (in && w) ? ((const float4*)w)[q] : make_float4(1.f, 1.f, 1.f, 1.f);
      }
    }
#pragma unroll
    for (int k = 0; k < B; ++k) {
      const int q = q0 + tid + k * T;
      if (k < step && q < (kp >> 2)) {
        float4 x = v[k];
        if (xown && 4 * q + 3 >= o0 && 4 * q < o1) {
          const float e[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (4 * q + c >= o0 && 4 * q + c < o1) xown[4 * q + c - o0] = e[c];
        }
        ss += (x.x * x.x + x.y * x.y) + (x.z * x.z + x.w * x.w);
        if (w) {
          x.x *= ww[k].x;
          x.y *= ww[k].y;
          x.z *= ww[k].z;
          x.w *= ww[k].w;
        }
        *(float4*)(vec + 4 * q) = x;
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

// One slot of a GEMV phase: rows [i, i + n) of the phase, whose first row is row g0 of the
// weight copy (the key of its unit swizzle). Each lane dots its units of its row, the lanes of
// a row are summed, and the warp's sum of row i + j goes to part[(i + j) * 8 + warp].
// U: the lane's units per row when known at compile time (all of them loaded before the first
// product), 0 for d.upl <= 8 at run time.
template <int U>
__device__ __forceinline__ void dec_slot(const uint8_t* slot, int n, int i, int g0, int kp,
                                         const DecLane& d, const float4 (&x)[16], float* part,
                                         int warp) {
  constexpr int UM = U ? U : 8;
  const bool mine = d.row < n;
  const int rr = mine ? d.row : 0;  // a lane without a row reads row 0 and drops the sum
  const uint8_t* row = slot + (size_t)rr * kp * 2;
  const int key = (g0 + i + rr) & 7;
  float2 a0 = make_float2(0.f, 0.f), a1 = a0;
  const auto dot = [&](const uint4& v, int t) {
    ffma2(a0, make_float2(bf16lo(v.x), bf16hi(v.x)), make_float2(x[2 * t].x, x[2 * t].y));
    ffma2(a1, make_float2(bf16lo(v.y), bf16hi(v.y)), make_float2(x[2 * t].z, x[2 * t].w));
    ffma2(a0, make_float2(bf16lo(v.z), bf16hi(v.z)), make_float2(x[2 * t + 1].x, x[2 * t + 1].y));
    ffma2(a1, make_float2(bf16lo(v.w), bf16hi(v.w)), make_float2(x[2 * t + 1].z, x[2 * t + 1].w));
  };
  if constexpr (U > 0) {
    uint4 v[UM];
#pragma unroll
    for (int t = 0; t < UM; ++t) v[t] = *(const uint4*)(row + (((d.u0 + d.us * t) ^ key) << 4));
#pragma unroll
    for (int t = 0; t < UM; ++t) dot(v[t], t);
  } else {
#pragma unroll
    for (int t = 0; t < UM; ++t)
      if (t < d.upl) dot(*(const uint4*)(row + (((d.u0 + d.us * t) ^ key) << 4)), t);
  }
  float s = (a0.x + a0.y) + (a1.x + a1.y);
  if (d.us == 1) {  // the lanes of a row are R apart
    for (int o = 32 / d.lpr; o < 32; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  } else {          // the lanes of a row are adjacent
    for (int o = d.lpr >> 1; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  }
  if (mine && d.sub == 0) part[(i + d.row) * kConsumerWarps + warp] = s;
}

// ---- GEMV slots on the tensor cores ------------------------------------------------------------
// For K up to 2048 a slot is done with mma.sync m16n8k16 (BF16 in, F32 accumulate): warp w
// takes the same columns [w kp / 8, (w + 1) kp / 8) = KS steps of 16, the weights of 16 rows x 16
// columns as A (ldmatrix from the swizzled row-major copy), and the phase's input as B with its
// hi part in column 0 and its lo part in column 1 (x = hi + lo to 2^-17, the split the per-layer
// GEMVs use), so D[r][0] + D[r][1] is the row's dot product over the warp's columns.
// B fragment of the lane (m16n8k16, "col" B): b0 = B[k][n], B[k + 1][n], b1 = the same at k + 8,
// with n = lane / 4 and k = 2 (lane % 4) of each 16-column step.
// The staged input (kp F32 values at vec) becomes its hi parts (BF16, vec[0 .. kp / 2) as
// floats) and lo parts (after them), in place: each value is split once per CTA.
__device__ __forceinline__ void dec_split_vec(float* vec, int kp, int tid) {
  constexpr int T = kConsumerWarps * 32;
  float v[8];  // kp <= 2048: at most 8 values a thread
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = tid + j * T < kp ? vec[tid + j * T] : 0.f;
  consumer_sync();
  uint16_t* hi = (uint16_t*)vec;
  uint16_t* lo = hi + kp;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (tid + j * T < kp) split_bf16(v[j], hi[tid + j * T], lo[tid + j * T]);
  consumer_sync();
}

template <int KS>
__device__ __forceinline__ void dec_load_xb(const float* vec, int kp, int warp, int lane,
                                            uint32_t (&xb)[KS][2]) {
  const int n = lane >> 2, kq = (lane & 3) * 2;
  const int c0 = warp * (kp >> 3);
  const uint16_t* src = (const uint16_t*)vec + (n == 1 ? kp : 0) + c0 + kq;  // hi or lo parts
#pragma unroll
  for (int t = 0; t < KS; ++t) {
    xb[t][0] = n < 2 ? *(const uint32_t*)(src + 16 * t) : 0u;
    xb[t][1] = n < 2 ? *(const uint32_t*)(src + 16 * t + 8) : 0u;
  }
}

// One slot of MT 16-row tiles (rows [i, i + n) of the phase, the first row g0 of the weight copy):
// the warp's partial sum of each row goes to part[row * 8 + warp]. Rows past n read row 0 and are
// dropped.
template <int KS, int MT>
__device__ __forceinline__ void dec_slot_mma(const uint8_t* slot, int n, int i, int g0, int kp,
                                             const uint32_t (&xb)[KS][2], float* part, int warp,
                                             int lane) {
  const int mi = lane >> 3;
  const int u0 = (warp * (kp >> 3)) >> 3;  // the warp's first 16-byte unit
  constexpr int NC = KS < 4 ? KS : 4;       // independent accumulator chains (k steps mod NC)
  float d[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    float c[NC][4];
#pragma unroll
    for (int j = 0; j < NC; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = 0.f;
    const int ra = mt * 16 + (mi & 1) * 8 + (lane & 7);
    const int rr = ra < n ? ra : 0;
    const uint8_t* row = slot + (size_t)rr * kp * 2;
    const int key = (g0 + i + rr) & 7;
#pragma unroll
    for (int t = 0; t < KS; ++t) {
      uint32_t af[4];
      ldmatrix_x4(af, row + (((u0 + 2 * t + (mi >> 1)) ^ key) << 4));
      mma_bf16(c[t % NC], af, xb[t][0], xb[t][1]);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float v = c[0][q];
#pragma unroll
      for (int j = 1; j < NC; ++j) v += c[j][q];
      d[mt][q] = v;
    }
  }
  if ((lane & 3) == 0) {
    const int g = lane >> 2;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      if (mt * 16 + g < n) part[(i + mt * 16 + g) * kConsumerWarps + warp] = d[mt][0] + d[mt][1];
      if (mt * 16 + g + 8 < n) part[(i + mt * 16 + g + 8) * kConsumerWarps + warp] = d[mt][2] + d[mt][3];
    }
  }
}

// The part table's rows summed in warp order, then epi for every row (or gate/up pair), one per
// thread (after the slots of a phase).
template <typename Epi>
__device__ __forceinline__ void dec_rows_epilogue(int rows, const float* part, int tid, bool pairs,
                                                  Epi&& epi) {
  consumer_sync();
  const int outs = pairs ? rows >> 1 : rows;
  for (int t = tid; t < outs; t += kConsumerWarps * 32) {
    const float4* p = (const float4*)(part + (size_t)(pairs ? 2 * t : t) * kConsumerWarps);
    const float4 a0 = p[0], a1 = p[1];
    const float v0 = ((a0.x + a0.y) + (a0.z + a0.w)) + ((a1.x + a1.y) + (a1.z + a1.w));
    float v1 = 0.f;
    if (pairs) {
      const float4 b0 = p[2], b1 = p[3];
      v1 = ((b0.x + b0.y) + (b0.z + b0.w)) + ((b1.x + b1.y) + (b1.z + b1.w));
    }
    epi(pairs ? 2 * t : t, v0, v1);
  }
}

// dec_rows on the tensor cores (slots of R <= 32 rows, K = 128 KS); the staged input at vec is
// split into its hi and lo parts in place first.
template <int KS, typename Epi>
__device__ __forceinline__ bool dec_rows_mma(DecRing& r, bool live, int rows, int g0, int kp, int R,
                                             float* vec, float* part, int warp, int lane,
                                             int tid, bool pairs, Epi&& epi) {
  uint32_t xb[KS][2];
  if (live) dec_split_vec(vec, kp, tid);
  dec_load_xb<KS>(vec, kp, warp, lane, xb);
  for (int i = 0; i < rows; i += R) {
    const int n = rows - i < R ? rows - i : R;
    if (!dec_take(r)) return false;
    if (live) {
      if (R > 16)
        dec_slot_mma<KS, 2>(r.cur(), n, i, g0, kp, xb, part, warp, lane);
      else
        dec_slot_mma<KS, 1>(r.cur(), n, i, g0, kp, xb, part, warp, lane);
    }
    dec_release(r, lane);
  }
  if (!live) return true;
  dec_rows_epilogue(rows, part, tid, pairs, epi);
  return true;
}

// Consumes one weight segment of `rows` rows (from row g0 of the weight copy) in slots of R,
// then sums the warps' partials of every row (in warp order) and runs epi(row, value, -) for
// every row — or, with pairs, epi(row, gate, up) for each gate/up pair (row, row + 1) — one
// row per thread. `live` false only releases the slots.
// `x` holds the lane's slice of the phase's input (dec_load_x), and `part` room for rows x 8
// floats.
template <typename Epi>
__device__ __forceinline__ bool dec_rows(DecRing& r, bool live, int rows, int g0, int kp, int R,
                                         const DecLane& d, const float4 (&x)[16], float* part,
                                         int warp, int lane, int tid, bool pairs, Epi&& epi) {
  for (int i = 0; i < rows; i += R) {
    const int n = rows - i < R ? rows - i : R;
    if (!dec_take(r)) return false;
    if (live) {
      switch (d.upl) {  // the units per lane of the Qwen3-0.6B phases: QKV and gate/up, down, O
        case 8: dec_slot<8>(r.cur(), n, i, g0, kp, d, x, part, warp); break;
        case 6: dec_slot<6>(r.cur(), n, i, g0, kp, d, x, part, warp); break;
        case 4: dec_slot<4>(r.cur(), n, i, g0, kp, d, x, part, warp); break;
        default: dec_slot<0>(r.cur(), n, i, g0, kp, d, x, part, warp); break;
      }
    }
    dec_release(r, lane);  // this warp's reads of the slot are done (the sums depend on them)
  }
  if (!live) return true;
  dec_rows_epilogue(rows, part, tid, pairs, epi);
  return true;
}

// A GEMV phase over the staged input `vec` (kp columns): on the tensor cores for kp = 256, 1024
// and 2048, on the CUDA cores otherwise. Measured on the Qwen3-0.6B step (2048 cached
// positions): the tensor cores for O (256) and QKV, gate/up (1024) with down (3072) on the CUDA
// cores 747 us, all on the CUDA cores 789 us, all four on the tensor cores 812 us.
template <typename Epi>
__device__ __forceinline__ bool dec_phase(DecRing& r, bool live, int rows, int g0, int kp, int R,
                                          float* vec, float* part, int warp, int lane,
                                          int tid, bool pairs, Epi&& epi) {
  switch (kp) {
    case 256: return dec_rows_mma<2>(r, live, rows, g0, kp, R, vec, part, warp, lane, tid, pairs, epi);
    case 1024: return dec_rows_mma<8>(r, live, rows, g0, kp, R, vec, part, warp, lane, tid, pairs, epi);
    case 2048: return dec_rows_mma<16>(r, live, rows, g0, kp, R, vec, part, warp, lane, tid, pairs, epi);
    default: {
      const DecLane d = dec_lane(kp, R, warp, lane);
      float4 x[16];
      dec_load_x(vec, d, x);
      return dec_rows(r, live, rows, g0, kp, R, d, x, part, warp, lane, tid, pairs, epi);
    }
  }
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
    target += (uint32_t)a.extra_arrivals;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t n = 1; ld_acquire_gpu(&a.sync[0]) < target; ++n) {
      if ((n & 63) == 0) {
        if (ld_acquire_gpu(&a.sync[1])) {
          ok = 0;
          break;
        }
        if (global_timer_ns() - t0 > a.wait_ns) {
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

// Online-softmax state of one lane group over its keys for G query heads: running max and
// sum, and the unnormalised output on the lane's 16 head dims.
template <int G>
struct DecAttnState {
  float m[G], l[G], o[G][16];
};

// One key for the lane's group: k/v are the lane's 16 dims, q its 16 dims of each query head;
// the eight lanes of the group hold the rest. `valid` false: the state does not change (the
// lanes still take part in the group's shuffles).
template <int G>
__device__ __forceinline__ void dec_attn_key(DecAttnState<G>& st, const float (&q)[G][16],
                                             const float (&k)[16], const float (&v)[16], bool valid,
                                             float inv_scale) {
  float sc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int e = 0; e < 16; e += 2)
      ffma2(acc, make_float2(q[g][e], q[g][e + 1]), make_float2(k[e], k[e + 1]));
    sc[g] = acc.x + acc.y;
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1)
#pragma unroll
    for (int g = 0; g < G; ++g) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], o);
  if (!valid) return;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float s = sc[g] * inv_scale;
    const float mn = fmaxf(st.m[g], s);
    const float al = __expf(st.m[g] - mn);  // 0 for the first key (m = -inf)
    const float p = __expf(s - mn);
    st.l[g] = st.l[g] * al + p;
#pragma unroll
    for (int e = 0; e < 16; ++e) st.o[g][e] = st.o[g][e] * al + p * v[e];
    st.m[g] = mn;
  }
}

// Two keys a then b for the lane's group: their scores are formed and reduced together (two
// independent chains), then the state takes key a and then key b exactly as two dec_attn_key
// calls would.
template <int G>
__device__ __forceinline__ void dec_attn_key2(DecAttnState<G>& st, const float (&q)[G][16],
                                              const float (&ka)[16], const float (&va)[16], bool va_ok,
                                              const float (&kb)[16], const float (&vb)[16], bool vb_ok,
                                              float inv_scale) {
  float sa[G], sb[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float2 acc = make_float2(0.f, 0.f), bcc = acc;
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
      ffma2(acc, make_float2(q[g][e], q[g][e + 1]), make_float2(ka[e], ka[e + 1]));
      ffma2(bcc, make_float2(q[g][e], q[g][e + 1]), make_float2(kb[e], kb[e + 1]));
    }
    sa[g] = acc.x + acc.y;
    sb[g] = bcc.x + bcc.y;
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      sa[g] += __shfl_xor_sync(0xffffffffu, sa[g], o);
      sb[g] += __shfl_xor_sync(0xffffffffu, sb[g], o);
    }
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    if (w == 0 ? !va_ok : !vb_ok) continue;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float s = (w == 0 ? sa[g] : sb[g]) * inv_scale;
      const float mn = fmaxf(st.m[g], s);
      const float al = __expf(st.m[g] - mn);  // 0 for the first key (m = -inf)
      const float p = __expf(s - mn);
      st.l[g] = st.l[g] * al + p;
#pragma unroll
      for (int e = 0; e < 16; ++e) st.o[g][e] = st.o[g][e] * al + p * (w == 0 ? va[e] : vb[e]);
      st.m[g] = mn;
    }
  }
}

// Attention unit (KV head h, split s) for the single query position pos: QK-RMSNorm + RoPE
// of the G query heads and of the new key (tiny.rs:24-37), the new K/V row written by the
// unit that holds pos, online softmax over the streamed cached rows (tiny.rs:77-101), the
// unit's partial (max, sum, output) per query head, and the merge of the head's S splits by
// every unit of the head once all are in. A key is taken by eight lanes: lane group
// kg = lane / 8 of warp w takes the keys 4 w + kg of each 32-key slot, lane q8 = lane % 8 the
// head dims of 16-byte units q8 and q8 + 8 (dims 8 q8 .. 8 q8 + 7 and 64 + 8 q8 .. 64 + 8 q8 + 7).
// Returns false when a ring slot never landed; *live_out false when the step was aborted.
template <int G>  // query heads per KV head (a.G)
__device__ __forceinline__ bool dec_attention(const DecodeArgs& a, const DecodeLayer& L,
                                              const DecPlan& P, DecRing& r, bool live, int pos,
                                              int layer, float* vec, float* ah,
                                              int* flag, bool* live_out, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int hd = kDecHd, half = hd / 2;
  const int h = P.h;
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
      // dims i and i + half, i = lane + 32 t.
      float x0[2], x1[2], w0[2], w1[2];
      float2 cs[2];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int i = lane + 32 * t;
        x0[t] = __ldcg(src + i);
        x1[t] = __ldcg(src + i + half);
        w0[t] = w[i];
        w1[t] = w[i + half];
        cs[t] = rp[i];
      }
      const float ssq = warp_sum((x0[0] * x0[0] + x1[0] * x1[0]) + (x0[1] * x0[1] + x1[1] * x1[1]));
      const float rms = sqrtf(ssq / (float)hd + a.eps);
      float* dst = isq ? qs + p * hd : kn;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int i = lane + 32 * t;
        const float y0 = x0[t] / rms * w0[t], y1 = x1[t] / rms * w1[t];
        dst[i] = y0 * cs[t].x - y1 * cs[t].y;
        dst[i + half] = y1 * cs[t].x + y0 * cs[t].y;
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
  const int kg = lane >> 3, q8 = lane & 7;
  // The lane's dims of every query head, and the group's state.
  float q[G][16];
  DecAttnState<G> st;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    st.m[g] = -INFINITY;
    st.l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      st.o[g][e] = 0.f;
      const int d = (e < 8 ? 8 * q8 : half + 8 * q8) + (e & 7);
      q[g][e] = live ? qs[g * hd + d] : 0.f;
    }
  }
  // The lane's 16 dims of one cache row j (hi + lo parts, kv_offset layout).
  auto load_row = [&](const uint8_t* row, int j, float (&out)[16]) {
#pragma unroll
    for (int hu = 0; hu < 2; ++hu) {
      const int u = (q8 + 8 * hu) ^ (j & 7);
      const uint4 hi = *(const uint4*)(row + (u << 4));
      const uint4 lo = *(const uint4*)(row + 2 * hd + (u << 4));
      float* o = out + 8 * hu;
      o[0] = bf16lo(hi.x) + bf16lo(lo.x);
      o[1] = bf16hi(hi.x) + bf16hi(lo.x);
      o[2] = bf16lo(hi.y) + bf16lo(lo.y);
      o[3] = bf16hi(hi.y) + bf16hi(lo.y);
      o[4] = bf16lo(hi.z) + bf16lo(lo.z);
      o[5] = bf16hi(hi.z) + bf16hi(lo.z);
      o[6] = bf16lo(hi.w) + bf16lo(lo.w);
      o[7] = bf16hi(hi.w) + bf16hi(lo.w);
    }
  };
  // Warps 0-3 take the even slots and warps 4-7 the odd ones, so two slots are worked on at
  // once; in its slots a lane group takes keys 4 (w % 4) + kg + 16 j (two at a time). Every
  // warp waits for every slot before releasing it (no warp runs a ring cycle ahead).
  const int npos = P.pe - P.p0;
  const int wh = warp >> 2, wq = warp & 3;
  for (int i0 = 0, si = 0; i0 < npos; i0 += P.kvps, ++si) {
    const int n = npos - i0 < P.kvps ? npos - i0 : P.kvps;
    if (!dec_take(r)) return false;
    if (live && (si & 1) == wh) {
      const uint8_t* ks = r.cur();
      const uint8_t* vs = ks + kDecKvHalf;
      for (int kk = 4 * wq + kg; kk - kg < n; kk += 32) {
        const int kb = kk + 16;
        const bool va = kk < n, vb = kb < n;
        const int ia = va ? kk : 0, ib = vb ? kb : 0;
        float k0[16], v0[16], k1[16], v1[16];
        load_row(ks + (size_t)ia * P.rowb, P.p0 + i0 + ia, k0);
        load_row(vs + (size_t)ia * P.rowb, P.p0 + i0 + ia, v0);
        load_row(ks + (size_t)ib * P.rowb, P.p0 + i0 + ib, k1);
        load_row(vs + (size_t)ib * P.rowb, P.p0 + i0 + ib, v1);
        dec_attn_key2<G>(st, q, k0, v0, va, k1, v1, vb, a.inv_scale);
      }
    }
    dec_release(r, lane);
  }
  if (!live) return true;
  if (P.has_new && warp == 0) {
    // The step's own key and value (F32, from the prologue), taken by lane group 0.
    float k[16], v[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int d = (e < 8 ? 8 * q8 : half + 8 * q8) + (e & 7);
      k[e] = kn[d];
      v[e] = vn[d];
    }
    dec_attn_key<G>(st, q, k, v, kg == 0, a.inv_scale);
  }
  // Merge the four lane groups of the warp (lanes q8, q8 + 8, q8 + 16, q8 + 24 hold the same
  // dims), then the warps' partials in shared memory.
#pragma unroll
  for (int o = 8; o < 32; o <<= 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mo = __shfl_xor_sync(0xffffffffu, st.m[g], o);
      const float lo = __shfl_xor_sync(0xffffffffu, st.l[g], o);
      const float M = fmaxf(st.m[g], mo);
      const float fa = st.m[g] == -INFINITY ? 0.f : __expf(st.m[g] - M);
      const float fb = mo == -INFINITY ? 0.f : __expf(mo - M);
      st.l[g] = st.l[g] * fa + lo * fb;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float oo = __shfl_xor_sync(0xffffffffu, st.o[g][e], o);
        st.o[g][e] = st.o[g][e] * fa + oo * fb;
      }
      st.m[g] = M;
    }
  }
  const int stride = hd + 4;
  if (kg == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float* mw = mrg + (size_t)(warp * G + g) * stride;
      if (q8 == 0) {
        mw[0] = st.m[g];
        mw[1] = st.l[g];
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) mw[4 + (e < 8 ? 8 * q8 : half + 8 * q8) + (e & 7)] = st.o[g][e];
    }
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
  // Every unit of the head waits for the head's S partials of this layer (the counter counts
  // the units of every layer so far), then merges all of them itself: exp(max_s - max)
  // weights in split order. The merged output (G query heads x head_dim) goes to `ah`, the
  // input vector of the O rows' phase.
  if (tid == 0) {
    int ok = 1;
    red_release_gpu(&a.sync[2 + h], 1u);
    const uint32_t target = (uint32_t)((layer + 1) * S);
    const uint64_t t0 = global_timer_ns();
    for (uint32_t n = 1; ld_acquire_gpu(&a.sync[2 + h]) < target; ++n) {
      if ((n & 63) == 0) {
        if (ld_acquire_gpu(&a.sync[1])) {
          ok = 0;
          break;
        }
        if (global_timer_ns() - t0 > a.wait_ns) {
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
  if (!*flag) {
    *live_out = false;
    return true;
  }
  float* Ms = mrg;           // [G][S] (the warps' partials are no longer needed)
  float* Ss = mrg + G * S;   // [G][S]
  // The thread's first output element's column of the S partials and the (max, sum) pairs go
  // out as one batch of loads (one L2 round trip).
  const auto column = [&](int e) { return a.part + (size_t)(h * G + e / hd) * S * stride + 4 + e % hd; };
  float pv[32];
  if (tid < G * hd) {
    const float* col = column(tid);
#pragma unroll
    for (int sp = 0; sp < 32; ++sp) pv[sp] = sp < S ? __ldcg(col + (size_t)sp * stride) : 0.f;
  }
  for (int e = tid; e < G * S; e += kConsumerWarps * 32) {
    const int g = e / S, sp = e - g * S;
    const float2 ml = __ldcg((const float2*)(a.part + ((size_t)(h * G + g) * S + sp) * stride));
    Ms[e] = ml.x;
    Ss[e] = ml.y;
  }
  consumer_sync();
  // The merge weight exp(max_s - max) of every (query head, split), formed once.
  float* Wf = Ss + G * S;  // [G][S]
  for (int e = tid; e < G * S; e += kConsumerWarps * 32) {
    const int g = e / S;
    float M = -INFINITY;
    for (int sp = 0; sp < S; ++sp) M = fmaxf(M, Ms[g * S + sp]);
    Wf[e] = Ms[e] == -INFINITY ? 0.f : expf(Ms[e] - M);
  }
  consumer_sync();
  for (int e = tid; e < G * hd; e += kConsumerWarps * 32) {
    const int g = e / hd;
    const float* col = column(e);
    if (e != tid) {
#pragma unroll
      for (int sp = 0; sp < 32; ++sp) pv[sp] = sp < S ? __ldcg(col + (size_t)sp * stride) : 0.f;
    }
    float Ls = 0.f, O = 0.f;
#pragma unroll
    for (int sp = 0; sp < 32; ++sp) {
      if (sp < S) {
        const float f = Wf[g * S + sp];
        Ls += Ss[g * S + sp] * f;
        O += pv[sp] * f;
      }
    }
    for (int sp = 32; sp < S; ++sp) {
      const float f = Wf[g * S + sp];
      Ls += Ss[g * S + sp] * f;
      O += __ldcg(col + (size_t)sp * stride) * f;
    }
    ah[e] = O / Ls;
  }
  consumer_sync();
  return true;
}

template <int G>  // query heads per KV head (a.G)
__global__ void __launch_bounds__(kDecThreads, 1) pp_decode_step_kernel(const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const int NG = gridDim.x, b = blockIdx.x, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int own_cap = (a.H + NG - 1) / NG + 1;
  const DecodeSmem lay(a.nslots, a.vec_floats, own_cap,
                       decode_part_rows(a.H, a.Q, a.KV, a.I, a.nkv, NG));
  DecRing r;
  r.base = smem;
  r.full = (uint64_t*)(smem + lay.bar_off());
  r.empty = r.full + a.nslots;
  r.ns = a.nslots;
  r.slot = 0;
  r.phase = 0;
  r.n = 0;
  float* vec = (float*)(smem + lay.vec_off());
  float* xown = (float*)(smem + lay.own_off());
  float* part = (float*)(smem + lay.part_off());
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
  if (warp >= kConsumerWarps) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kDecProducerRegs));
    if (warp != kConsumerWarps || lane != 0) return;
    bool ok = true;
    for (int l = 0; l < a.nl && ok; ++l) {
      const DecodeLayer& L = a.layers[l];
      ok = dec_issue_rows(r, L.wqkv + (size_t)P.q0 * a.kH, P.q1 - P.q0, a.kH * 2, P.rps_qkv);
      if (ok && P.h >= 0) {
        const size_t off = ((size_t)P.h * a.capacity + P.p0) * P.rowb;
        ok = dec_issue_kv(r, L.kc + off, L.vc + off, P.pe - P.p0, P.rowb, P.kvps);
      }
      if (ok && P.h >= 0)
        ok = dec_issue_rows(r, L.wo + ((size_t)P.h * a.H + P.r0) * a.kO, P.r1 - P.r0, a.kO * 2,
                            P.rps_oh);
      ok = ok && dec_issue_rows(r, L.wgu + (size_t)2 * P.j0 * a.kH, 2 * (P.j1 - P.j0), a.kH * 2, P.rps_gu);
      ok = ok && dec_issue_rows(r, L.wd + (size_t)P.o0 * a.kI, P.o1 - P.o0, a.kI * 2, P.rps_d);
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
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kDecConsumerRegs));
  // Per layer, four grid barriers and one barrier among the units of each KV head:
  //   QKV (input RMSNorm) | attention: each unit's partial, the head's units meet, every unit
  //   merges the head's splits and computes its rows of the head's share of O | gate/up (the
  //   residual plus every head's share of O, the post-attention RMSNorm, SwiGLU) | down +
  //   residual |
  bool live = true, lost = false;  // lost: a ring slot never landed
  uint32_t nb = 0;
  float* ah = vec + decode_att_floats(a.hd, G);  // a head's merged attention output
  for (int l = 0; l < a.nl && !lost; ++l) {
    const DecodeLayer& L = a.layers[l];
    // ---- QKV with the input RMSNorm; layer 0 gathers the token's embedding row
    // (src/qwen/model.rs:239-241), also the first residual.
    {
      float rinv = 1.f;
      if (live) {
        float ss;
        if (l == 0) {
          float t = 0.f;
          for (int q = tid; q < (a.kH >> 2); q += kConsumerWarps * 32) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (q < (a.H >> 2)) {
              v.x = __uint_as_float((uint32_t)a.embed[tiled_offset(tok, 4 * q + 0, a.embed_kchunks)] << 16);
              v.y = __uint_as_float((uint32_t)a.embed[tiled_offset(tok, 4 * q + 1, a.embed_kchunks)] << 16);
              v.z = __uint_as_float((uint32_t)a.embed[tiled_offset(tok, 4 * q + 2, a.embed_kchunks)] << 16);
              v.w = __uint_as_float((uint32_t)a.embed[tiled_offset(tok, 4 * q + 3, a.embed_kchunks)] << 16);
              const int n0 = 4 * q;
              if (n0 + 3 >= P.o0 && n0 < P.o1) {  // the residual of this CTA's rows
                const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int c = 0; c < 4; ++c)
                  if (n0 + c >= P.o0 && n0 + c < P.o1) a.x[n0 + c] = e[c];
              }
              t += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
              const float4 ww = ((const float4*)L.n_attn)[q];
              v.x *= ww.x;
              v.y *= ww.y;
              v.z *= ww.z;
              v.w *= ww.w;
            }
            *(float4*)(vec + 4 * q) = v;
          }
          t = warp_sum(t);
          if (lane == 0) red[warp] = t;
          consumer_sync();
          ss = 0.f;
#pragma unroll
          for (int i = 0; i < kConsumerWarps; ++i) ss += red[i];
          consumer_sync();
        } else {
          ss = dec_stage_vec(a.x, nullptr, 0, L.n_attn, a.H, a.kH, vec, red, tid, nullptr, 0, 0);
        }
        rinv = 1.0f / sqrtf(ss / (float)a.H + a.eps);
      }
      if (!dec_phase(r, live, P.q1 - P.q0, P.q0, a.kH, P.rps_qkv, vec, part, warp, lane, tid,
                     false, [&](int rr, float v, float) { a.qkv[P.q0 + rr] = v * rinv; })) {
        lost = true;
        break;
      }
    }
    live = live && dec_grid_sync(a, ++nb * (uint32_t)NG, flag, tid);
    // ---- attention, then this unit's rows of its head's share of O (src/qwen/model.rs:304).
    if (P.h >= 0) {
      bool hlive = live;
      if (!dec_attention<G>(a, L, P, r, live, pos, l, vec, ah, flag, &hlive, tid)) {
        lost = true;
        break;
      }
      live = hlive;
      float* op = a.opart + (size_t)P.h * a.H + P.r0;
      if (!dec_phase(r, live, P.r1 - P.r0, P.r0, a.kO, P.rps_oh, ah, part, warp, lane, tid,
                     false, [&](int rr, float v, float) { op[rr] = v; })) {
        lost = true;
        break;
      }
    }
    live = live && dec_grid_sync(a, ++nb * (uint32_t)NG, flag, tid);
    // ---- gate/up: the residual after the attention (x plus every head's share of O; this
    // CTA keeps its own rows), the post-attention RMSNorm, SwiGLU (tiny.rs:111-115).
    {
      float rinv = 1.f;
      if (live) {
        const float ss = dec_stage_vec(a.x, a.opart, a.nkv, L.n_ffn, a.H, a.kH, vec, red, tid,
                                       xown, P.o0, P.o1);
        rinv = 1.0f / sqrtf(ss / (float)a.H + a.eps);
      }
      if (!dec_phase(r, live, 2 * (P.j1 - P.j0), 2 * P.j0, a.kH, P.rps_gu, vec, part, warp, lane,
                     tid, true, [&](int rr, float g, float u) {
                      g *= rinv;
                      u *= rinv;
                      a.act[P.j0 + (rr >> 1)] = g / (1.0f + expf(-g)) * u;
                    })) {
        lost = true;
        break;
      }
    }
    live = live && dec_grid_sync(a, ++nb * (uint32_t)NG, flag, tid);
    // ---- down + residual.
    {
      if (live) dec_stage_vec(a.act, nullptr, 0, nullptr, a.I, a.kI, vec, red, tid, nullptr, 0, 0);
      if (!dec_phase(r, live, P.o1 - P.o0, P.o0, a.kI, P.rps_d, vec, part, warp, lane, tid, false,
                     [&](int rr, float v, float) {
                      v += xown[rr];
                      xown[rr] = v;
                      a.x[P.o0 + rr] = v;
                    })) {
        lost = true;
        break;
      }
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

// The O projection regrouped per KV head for the decode kernel: block h is [H][kO] (the head's
// G query heads' kO = G * head_dim columns of W_o), dec_w_offset layout.
__global__ void pp_untile_o_heads_kernel(uint16_t* dst, const uint16_t* src, int64_t H, int64_t kO,
                                         int64_t nkv, int64_t kchunks) {
  const int64_t per = H * kO, n = nkv * per;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t h = i / per, rem = i - h * per, r = rem / kO, c = rem - r * kO;
    dst[h * per + dec_w_offset(r, c, kO)] = src[tiled_offset(r, h * kO + c, kchunks)];
  }
}

// Decode weight copies of the packed weights: dst row r of kp columns (dec_w_offset layout,
// zero past `cols`) = W[row(r)] with row(r) = r (QKV, O, down) or, for the gate/up pairs
// (mode 1), gate row r/2 or up row r/2 of the 64-row interleaved blocks.
__global__ void pp_untile_rows_kernel(uint16_t* dst, const uint16_t* src, int64_t rows, int64_t cols,
                                      int64_t kp, int64_t kchunks, int32_t mode) {
  const int64_t n = rows * kp;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / kp, c = i - r * kp;
    int64_t pr = r;
    if (mode == 1) {
      const int64_t j = r >> 1;
      pr = (j / (kTileRows / 2)) * kTileRows + (j % (kTileRows / 2)) + (r & 1) * (kTileRows / 2);
    }
    dst[dec_w_offset(r, c, kp)] = c < cols ? src[tiled_offset(pr, c, kchunks)] : (uint16_t)0;
  }
}

}  // namespace pp
