// Row kernels of the prompt prefill (pp_shard_prefill): the pieces between the tcgen05
// projections (pp_rows_gemm) when a whole prompt chunk of t rows goes through the layers at
// once. Rows are F32 with a row stride equal to their width. The arithmetic is the verify
// pass's: RMSNorm x * (1 / sqrt(mean(x^2) + eps)) * w (tiny.rs:20-23), per-head QK-norm and
// rotate-half RoPE at the absolute position with the K/V rows written into the cache
// (model.rs:267-302, tiny.rs:24-37), SwiGLU g / (1 + e^-g) * u (tiny.rs:111-115).
#pragma once
#include "pp_attn.cuh"
#include "pp_common.cuh"

namespace pp {

// x[t][c] = embedding row of tokens[t] (BF16 decoded), c < h; grid (t), 256 threads.
__global__ void pre_embed_kernel(const uint16_t* table, int32_t kchunks, const int32_t* tokens,
                                 int32_t h, float* x) {
  const int t = blockIdx.x, tok = tokens[t];
  for (int c = threadIdx.x; c < h; c += blockDim.x)
    x[(size_t)t * h + c] = __uint_as_float((uint32_t)table[tiled_offset(tok, c, kchunks)] << 16);
}

// y[t][c] = x[t][c] * (1 / sqrt(mean_c x[t][c]^2 + eps)) * w[c]; grid (t), 256 threads.
__global__ void pre_rmsnorm_kernel(const float* x, const float* w, int32_t h, float eps, float* y) {
  __shared__ float red[8];
  const float* xr = x + (size_t)blockIdx.x * h;
  float ss = 0.f;
  for (int c = threadIdx.x; c < h; c += blockDim.x) ss += xr[c] * xr[c];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
  const float rinv = 1.0f / sqrtf(t / (float)h + eps);
  float* yr = y + (size_t)blockIdx.x * h;
  for (int c = threadIdx.x; c < h; c += blockDim.x) yr[c] = xr[c] * rinv * w[c];
}

// x[i] += d[i] for i < n (the residual adds after O and down); grid-stride.
__global__ void pre_add_kernel(float* x, const float* d, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    x[i] += d[i];
}

// Projections qkv[t][Q + 2 KV] of rows at positions pos + t: per head RMSNorm with q_norm /
// k_norm and RoPE, queries to q[t][Q], keys and values into the cache rows of their heads.
// Grid (t, n_heads + 2 n_kv), one thread per dim pair (hd / 2 threads, hd <= 128).
__global__ void pre_qkv_kernel(const float* qkv, int32_t t_rows, int32_t pos, int32_t nh,
                               int32_t nkv, int32_t hd, float eps, const float* qn, const float* kn,
                               const float2* rope, uint8_t* kc, uint8_t* vc, int32_t capacity,
                               float* q) {
  __shared__ float red[4];
  const int t = blockIdx.x, head = blockIdx.y, i = threadIdx.x, half = hd >> 1;
  const int Q = nh * hd, KV = nkv * hd;
  const float* src = qkv + (size_t)t * (Q + 2 * KV) + (size_t)head * hd;
  const int p = pos + t;
  if (head >= nh + nkv) {  // value row
    uint8_t* row = vc + ((size_t)(head - nh - nkv) * capacity + p) * kv_row_bytes(hd);
    if (i < half) {
      kv_store(row, p, i, hd, src[i]);
      kv_store(row, p, i + half, hd, src[i + half]);
    }
    return;
  }
  const float x0 = i < half ? src[i] : 0.f, x1 = i < half ? src[i + half] : 0.f;
  float ss = warp_sum(x0 * x0 + x1 * x1);
  if ((i & 31) == 0) red[i >> 5] = ss;
  __syncthreads();
  ss = 0.f;
  for (int w = 0; w < (int)((blockDim.x + 31) >> 5); ++w) ss += red[w];
  if (i >= half) return;
  const float rms = sqrtf(ss / (float)hd + eps);
  const bool isq = head < nh;
  const float* w = isq ? qn : kn;
  const float y0 = x0 / rms * w[i], y1 = x1 / rms * w[i + half];
  const float2 cs = rope[(size_t)p * half + i];
  const float o0 = y0 * cs.x - y1 * cs.y, o1 = y1 * cs.x + y0 * cs.y;
  if (isq) {
    float* dst = q + (size_t)t * Q + (size_t)head * hd;
    dst[i] = o0;
    dst[i + half] = o1;
  } else {
    uint8_t* row = kc + ((size_t)(head - nh) * capacity + p) * kv_row_bytes(hd);
    kv_store(row, p, i, hd, o0);
    kv_store(row, p, i + half, hd, o1);
  }
}

// SwiGLU over the packed gate/up output (64-row blocks: gate rows then up rows of each 128):
// act[t][j] = g / (1 + e^-g) * u, j < I; grid-stride over t * I.
__global__ void pre_swiglu_kernel(const float* gu, int32_t gu_rows, int32_t I, int64_t t_rows,
                                  float* act) {
  const int64_t n = t_rows * I;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / I;
    const int j = (int)(e - t * I);
    const int pg = (j >> 6) * 128 + (j & 63);
    const float g = gu[t * gu_rows + pg], u = gu[t * gu_rows + pg + 64];
    act[e] = g / (1.0f + expf(-g)) * u;
  }
}

// Attention of every 16-row sub-chunk of a prompt chunk in one launch: grid
// (n_kv, splits, chunks); CTA (KV head h, split s, sub-chunk z) runs the split kernel's unit
// with the sub-chunk's step header descs[z], its query rows q + 16 z rows and its partials at
// part + z part_stride ([n_kv][splits][nq_max][4 + hd] per sub-chunk). A split past the keys of
// its sub-chunk writes an empty partial (max -inf, sum 0). The last sub-chunks see the most
// keys, so they take the lowest block indices and start first.
template <int NT>
__global__ void __launch_bounds__(kAttnThreads) pre_attn_kernel(const AttnArgs a,
                                                                const StepDesc* descs,
                                                                size_t part_stride) {
  extern __shared__ uint8_t attn_smem_raw[];
  uint8_t* sm = (uint8_t*)(((uintptr_t)attn_smem_raw + 127) & ~(uintptr_t)127);
  const AttnSmem L(a.head_dim, NT, kAttnStages);
  AttnArgs az = a;
  const int z = gridDim.z - 1 - blockIdx.z;
  az.desc = descs + z;
  az.q = a.q + (size_t)z * 16 * a.q_dim;
  az.part = a.part + (size_t)z * part_stride;
  if (bad_step(az.desc, az.capacity, 16)) return;
  if (threadIdx.x == 0) attn_init_barriers(L, sm);
  consumer_sync();  // barrier init visible to every thread
  uint32_t uses = 0;
  attn_unit<16, NT>(az, blockIdx.x, blockIdx.y, L, sm, uses);
}

// Merge of the splits of (query head hq, row r) of sub-chunk z into F32 rows
// out[16 z + r][hq * hd + d] (the combine of attn_combine_kernel with a row-major F32 output
// for the projection that follows). Grid (n_heads, 16, chunks), block max(32, hd).
__global__ void pre_attn_combine_kernel(const AttnArgs a, const StepDesc* descs,
                                        size_t part_stride, float* out, int32_t ldo) {
  const int hq = blockIdx.x, r = blockIdx.y, z = blockIdx.z;
  if (bad_step(descs + z, a.capacity, 16) || r >= descs[z].m) return;
  __shared__ float sm_m[64], sm_w[64];
  __shared__ float red_l;
  const int G = a.n_heads / a.n_kv;
  const int h = hq / G, g = hq - h * G;
  const int hd = a.head_dim, t = threadIdx.x, S = a.splits;
  const size_t stride = (size_t)a.nq_max * (hd + 4);
  const float* base = a.part + (size_t)z * part_stride +
                      ((size_t)h * S * a.nq_max + (size_t)(g * 16 + r)) * (hd + 4);
  for (int s = t; s < S; s += blockDim.x) {
    const float2 ml = __ldcg((const float2*)(base + s * stride));
    sm_m[s] = ml.x;
    sm_w[s] = ml.y;
  }
  __syncthreads();
  if (t == 0) {
    float mx = -INFINITY;
    for (int s = 0; s < S; ++s) mx = fmaxf(mx, sm_m[s]);
    float l = 0.f;
    for (int s = 0; s < S; ++s) {
      const float f = (sm_m[s] == -INFINITY) ? 0.f : expf(sm_m[s] - mx);
      l += sm_w[s] * f;
      sm_w[s] = f;
    }
    red_l = l;
  }
  __syncthreads();
  if (t < hd) {
    float o = 0.f;
    for (int s = 0; s < S; ++s) o += __ldcg(base + s * stride + 4 + t) * sm_w[s];
    out[(size_t)(16 * z + r) * ldo + hq * hd + t] = o / red_l;
  }
}

}  // namespace pp
