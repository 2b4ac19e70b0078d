// Causal GQA attention of the verify chunk against the shard's KV cache
// (src/qwen/model.rs:282-302 `paged_attention` + `causal_bias`; the scalar statement is
// src/qwen/tiny.rs:77-101): for the query row at absolute position p = pos + r,
//   out = softmax(q . k_j / sqrt(head_dim), j = 0..p) . v_j
// Keys 0..pos-1 were written by earlier steps, keys pos..pos+m-1 by this step's QKV epilogue;
// rows past pos+m-1 (a rejected speculative tail) are never read, which is the reference's
// rollback-by-overwrite.
//
// Split-KV decode layout: one CTA per (KV head, key range). All G*m query vectors that share
// the KV head (G = n_heads / n_kv_heads) are processed together so every K/V byte is read
// once per step; K/V tiles of 32 keys are double-buffered with cp.async; softmax is online
// (running max, rescaled sum). A second kernel merges the per-split partials.
#pragma once
#include "pp_common.cuh"

namespace pp {

struct AttnArgs {
  const float* q;       // [MT][q_dim], normed and rotated
  const float* kcache;  // [n_kv][capacity][head_dim]
  const float* vcache;
  float* part;          // [n_kv][splits][nq_max][head_dim + 2]
  uint8_t* out_split;   // attention output rows, split BF16 layout (input of the O GEMV)
  int32_t n_heads, n_kv, head_dim, capacity, splits, q_dim, nq_max;
  float scale;  // sqrt(head_dim); scores are divided by it as in tiny.rs:90
  const StepDesc* desc;
  StepResult* res;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kAttnStages = 3;  // K/V tiles in flight per CTA (cp.async groups)

// Shared memory (floats): qs[32][hdp] | K[S][32][hdp] | V[S][32][hdp] | ps[32][32] | st[3][32]
__host__ __device__ inline size_t attn_smem_bytes(int hd) {
  const int hdp = hd + 4;
  return (size_t)(32 * hdp + 2 * kAttnStages * kAttnTile * hdp + 32 * kAttnTile + 3 * 32) * 4;
}

template <int MT>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const AttnArgs a) {
  extern __shared__ float sm[];
  const int hd = a.head_dim, hdp = hd + 4;
  float* qs = sm;
  float* ks = qs + 32 * hdp;
  float* vs = ks + kAttnStages * kAttnTile * hdp;
  float* ps = vs + kAttnStages * kAttnTile * hdp;
  float* st_m = ps + 32 * kAttnTile;
  float* st_l = st_m + 32;

  const int tid = threadIdx.x;
  const int h = blockIdx.x, s = blockIdx.y;
  if (tid == 0) pdl_launch_dependents();
  if (bad_step(a.desc, a.capacity, MT)) return;
  pdl_wait();
  const int pos = a.desc->pos, m = a.desc->m;
  const int G = a.n_heads / a.n_kv;
  const int nq = G * MT;
  const int c = pos + m;  // keys visible to the last row
  const int ntiles = (c + kAttnTile - 1) / kAttnTile;
  const int tps = (ntiles + a.splits - 1) / a.splits;
  const int t0 = s * tps, t1 = min(ntiles, t0 + tps);
  const int kend = min(c, t1 * kAttnTile);  // this split covers keys [t0*32, kend)

  // Query vectors of this KV head: qi = g * MT + r, head h*G + g, row r.
  for (int e = tid; e < nq * hd; e += kAttnThreads) {
    const int qi = e / hd, dd = e - qi * hd;
    const int g = qi / MT, r = qi - g * MT;
    qs[qi * hdp + dd] = (r < m) ? a.q[(size_t)r * a.q_dim + (h * G + g) * hd + dd] : 0.f;
  }
  if (tid < 32) {
    st_m[tid] = -INFINITY;
    st_l[tid] = 0.f;
  }

  const float* kbase = a.kcache + (size_t)h * a.capacity * hd;
  const float* vbase = a.vcache + (size_t)h * a.capacity * hd;
  const int c4 = hd / 4;
  auto load_tile = [&](int buf, int tile) {
    const int j0 = tile * kAttnTile;
    float* kd = ks + buf * kAttnTile * hdp;
    float* vd = vs + buf * kAttnTile * hdp;
    for (int e = tid; e < kAttnTile * c4; e += kAttnThreads) {
      const int row = e / c4, col = (e - row * c4) * 4;
      const int jg = j0 + row;
      if (jg < kend) {
        cp_async16(kd + row * hdp + col, kbase + (size_t)jg * hd + col);
        cp_async16(vd + row * hdp + col, vbase + (size_t)jg * hd + col);
      } else {
        *(float4*)(kd + row * hdp + col) = make_float4(0.f, 0.f, 0.f, 0.f);
        *(float4*)(vd + row * hdp + col) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    cp_async_commit();
  };

  const int qi = tid >> 3, kg = tid & 7;
  const int g_q = qi / MT, r_q = qi - g_q * MT;
  const bool qvalid = qi < nq && r_q < m;
  const int p_q = pos + r_q;  // absolute position of this query row
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;

  // kAttnStages - 1 tiles in flight ahead of the one being computed; every iteration
  // commits exactly one (possibly empty) group so the wait count stays uniform.
#pragma unroll
  for (int i = 0; i < kAttnStages - 1; ++i) {
    if (t0 + i < t1)
      load_tile(i, t0 + i);
    else
      cp_async_commit();
  }
  for (int tile = t0; tile < t1; ++tile) {
    const int buf = (tile - t0) % kAttnStages;
    const int nxt = tile + kAttnStages - 1;
    if (nxt < t1)
      load_tile((nxt - t0) % kAttnStages, nxt);
    else
      cp_async_commit();
    cp_async_wait<kAttnStages - 1>();
    __syncthreads();
    const float* kt = ks + buf * kAttnTile * hdp;
    const float* vt = vs + buf * kAttnTile * hdp;
    // Scores: query qi against keys kg + 8i.
    float sc[4];
    {
      float2 dacc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) dacc[i] = make_float2(0.f, 0.f);
      const float* qrow = qs + (qi < 32 ? qi : 0) * hdp;
      for (int dd = 0; dd < hd; dd += 4) {
        const float4 qv = *(const float4*)(qrow + dd);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 kv = *(const float4*)(kt + (kg + 8 * i) * hdp + dd);
          ffma2(dacc[i], make_float2(qv.x, qv.y), make_float2(kv.x, kv.y));
          ffma2(dacc[i], make_float2(qv.z, qv.w), make_float2(kv.z, kv.w));
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int jg = tile * kAttnTile + kg + 8 * i;
        const bool vis = qvalid && jg < kend && jg <= p_q;
        sc[i] = vis ? (dacc[i].x + dacc[i].y) / a.scale : -INFINITY;
      }
    }
    float tmax = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
    tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 4));
    const float m_old = (qi < 32) ? st_m[qi] : -INFINITY;
    const float m_new = fmaxf(m_old, tmax);
    float psum = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float p = (sc[i] == -INFINITY) ? 0.f : expf(sc[i] - m_new);
      psum += p;
      if (qi < 32) ps[qi * kAttnTile + kg + 8 * i] = p;
    }
    psum += __shfl_xor_sync(0xffffffffu, psum, 1);
    psum += __shfl_xor_sync(0xffffffffu, psum, 2);
    psum += __shfl_xor_sync(0xffffffffu, psum, 4);
    const float alpha = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
    __syncthreads();  // everyone has read st_m before it changes
    if (kg == 0 && qi < 32) {
      st_m[qi] = m_new;
      st_l[qi] = st_l[qi] * alpha + psum;
    }
    // P.V: dims {4*kg + 32*i + e}.
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] *= alpha;
    if (qi < nq) {
      const float* prow = ps + qi * kAttnTile;
      for (int j = 0; j < kAttnTile; ++j) {
        const float p = prow[j];
        const float* vr = vt + j * hdp;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int dd = 4 * kg + 32 * i;
          if (dd < hd) {
            const float4 vv = *(const float4*)(vr + dd);
            acc[4 * i + 0] += p * vv.x;
            acc[4 * i + 1] += p * vv.y;
            acc[4 * i + 2] += p * vv.z;
            acc[4 * i + 3] += p * vv.w;
          }
        }
      }
    }
    __syncthreads();  // this buffer is refilled kAttnStages - 1 iterations later
  }
  cp_async_wait<0>();

  __syncthreads();
  // Partial of this split: running max, running sum, unnormalised output.
  if (qi < nq) {
    float* dst = a.part + (((size_t)h * a.splits + s) * a.nq_max + qi) * (hd + 2);
    if (kg == 0) {
      dst[0] = st_m[qi];
      dst[1] = st_l[qi];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int dd = 4 * kg + 32 * i;
      if (dd < hd) {
        dst[2 + dd + 0] = acc[4 * i + 0];
        dst[2 + dd + 1] = acc[4 * i + 1];
        dst[2 + dd + 2] = acc[4 * i + 2];
        dst[2 + dd + 3] = acc[4 * i + 3];
      }
    }
  }
}

// Merge the splits of one (query head, row): grid (n_heads, m), one thread per dimension.
template <int MT>
__global__ void attn_combine_kernel(const AttnArgs a) {
  if (threadIdx.x == 0) pdl_launch_dependents();
  if (bad_step(a.desc, a.capacity, MT)) return;
  pdl_wait();
  const int hq = blockIdx.x, r = blockIdx.y;
  if (r >= a.desc->m) return;
  const int G = a.n_heads / a.n_kv;
  const int h = hq / G, g = hq - h * G;
  const int qi = g * MT + r;
  const int hd = a.head_dim;
  const size_t stride = (size_t)a.nq_max * (hd + 2);
  const float* base = a.part + ((size_t)h * a.splits * a.nq_max + qi) * (hd + 2);
  // Per-split (max, sum) pairs are read once into shared memory with independent loads.
  __shared__ float sm_m[256], sm_w[256];
  __shared__ float red_l;
  const int S = a.splits;
  for (int s = threadIdx.x; s < S; s += blockDim.x) {
    sm_m[s] = __ldcg(base + s * stride);
    sm_w[s] = __ldcg(base + s * stride + 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mx = -INFINITY;
    for (int s = 0; s < S; ++s) mx = fmaxf(mx, sm_m[s]);
    float l = 0.f;
    for (int s = 0; s < S; ++s) {
      const float f = (sm_m[s] == -INFINITY) ? 0.f : expf(sm_m[s] - mx);
      l += sm_w[s] * f;
      sm_w[s] = f;  // now the scale of split s
    }
    red_l = l;
  }
  __syncthreads();
  const float inv_l = 1.0f / red_l;
  for (int dd = threadIdx.x; dd < hd; dd += blockDim.x) {
    float o = 0.f;
    for (int s0 = 0; s0 < S; s0 += 8) {
      float pv[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        pv[q] = (s0 + q < S && sm_w[s0 + q] != 0.f) ? __ldcg(base + (s0 + q) * stride + 2 + dd) : 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (s0 + q < S) o += pv[q] * sm_w[s0 + q];
    }
    store_split<MT>(a.out_split, r, hq * hd + dd, o * inv_l);
  }
}

}  // namespace pp
