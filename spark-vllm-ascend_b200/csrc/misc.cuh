// misc.cuh -- Q4_0 format kernels, standalone elementwise stages and decode bookkeeping.
#pragma once

#include "common.cuh"

namespace spark {

// ------------------------------------------------------------------ Q4_0 quantize
// One thread per 32-weight block; restates gguf 0.19.0 quants.Q4_0.quantize_blocks:
// signed absmax (first index on ties), d = max / -8, id = 1 / d (0 if d == 0),
// q = clip(trunc(w * id + 8.5), 0, 15), byte j = q[j] | q[j+16] << 4, d -> fp16 (RNE).
__global__ void q4_quantize_kernel(const float* __restrict__ w, int64_t nblocks, uint8_t* __restrict__ qs,
                                   uint16_t* __restrict__ d) {
  for (int64_t blk = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; blk < nblocks;
       blk += (int64_t)gridDim.x * blockDim.x) {
    const float4* src = reinterpret_cast<const float4*>(w + blk * 32);
    float v[32];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      float4 t = src[i];
      v[4 * i] = t.x;
      v[4 * i + 1] = t.y;
      v[4 * i + 2] = t.z;
      v[4 * i + 3] = t.w;
    }
    int imax = 0;
    float amax = fabsf(v[0]);
#pragma unroll
    for (int j = 1; j < 32; j++) {
      float a = fabsf(v[j]);
      if (a > amax) {
        amax = a;
        imax = j;
      }
    }
    float mx = v[0];
#pragma unroll
    for (int j = 1; j < 32; j++)
      if (j == imax) mx = v[j];
    const float dd = __fdiv_rn(mx, -8.0f);
    const float id = (dd == 0.0f) ? 0.0f : __fdiv_rn(1.0f, dd);
    uint32_t words[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 16; j++) {
      int lo = (int)truncf(__fadd_rn(__fmul_rn(v[j], id), 8.5f));
      int hi = (int)truncf(__fadd_rn(__fmul_rn(v[j + 16], id), 8.5f));
      lo = lo > 15 ? 15 : (lo < 0 ? 0 : lo);
      hi = hi > 15 ? 15 : (hi < 0 ? 0 : hi);
      words[j >> 2] |= (uint32_t)(lo | (hi << 4)) << (8 * (j & 3));
    }
    // qs row layout == block-major within a row, so block blk's bytes are at blk*16
    *reinterpret_cast<uint4*>(qs + blk * 16) = make_uint4(words[0], words[1], words[2], words[3]);
    d[blk] = __half_as_ushort(__float2half_rn(dd));
  }
}

// gguf bytes [nblocks][18] -> planes
__global__ void q4_split_kernel(const uint8_t* __restrict__ blocks, int64_t nblocks, uint8_t* __restrict__ qs,
                                uint16_t* __restrict__ d) {
  for (int64_t blk = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; blk < nblocks;
       blk += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t* src = blocks + blk * 18;
    d[blk] = (uint16_t)(src[0] | (src[1] << 8));
    uint32_t words[4];
#pragma unroll
    for (int i = 0; i < 4; i++)
      words[i] = (uint32_t)src[2 + 4 * i] | ((uint32_t)src[3 + 4 * i] << 8) | ((uint32_t)src[4 + 4 * i] << 16) |
                 ((uint32_t)src[5 + 4 * i] << 24);
    *reinterpret_cast<uint4*>(qs + blk * 16) = make_uint4(words[0], words[1], words[2], words[3]);
  }
}

__global__ void q4_dequant_bf16_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ d, int64_t nblocks,
                                       uint16_t* __restrict__ w) {
  for (int64_t blk = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; blk < nblocks;
       blk += (int64_t)gridDim.x * blockDim.x) {
    const float s = h2f(d[blk]);
    const uint4 q = *reinterpret_cast<const uint4*>(qs + blk * 16);
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
    uint16_t* o = w + blk * 32;
#pragma unroll
    for (int j = 0; j < 16; j++) {
      uint32_t byte = (words[j >> 2] >> (8 * (j & 3))) & 0xffu;
      o[j] = f2bf(__fmul_rn(s, (float)((int)(byte & 15u) - 8)));
      o[j + 16] = f2bf(__fmul_rn(s, (float)((int)(byte >> 4) - 8)));
    }
  }
}

// ------------------------------------------------------------------ standalone add + RMSNorm
// One CTA of 1024 threads; same canonical order as the GEMV prologue.
__global__ void __launch_bounds__(1024) add_rmsnorm_kernel(const uint16_t* __restrict__ a,
                                                           const uint16_t* __restrict__ b,
                                                           const uint16_t* __restrict__ gamma, float eps, float inv_h,
                                                           int h, uint16_t* res_out, uint16_t* y) {
  extern __shared__ float s_sm[];
  __shared__ float inv_s;
  pdl_launch_dependents();
  pdl_wait();
  for (int i = threadIdx.x; i < h; i += blockDim.x) {
    float s = b ? __fadd_rn(bf2f(a[i]), bf2f(b[i])) : bf2f(a[i]);
    s_sm[i] = s;
    if (res_out) res_out[i] = f2bf(s);
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    float acc = 0.0f;
    for (int i = threadIdx.x; i < h; i += 32) acc = __fadd_rn(acc, __fmul_rn(s_sm[i], s_sm[i]));
    acc = butterfly_sum<32>(acc);
    if (threadIdx.x == 0) inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(acc, inv_h), eps)));
  }
  __syncthreads();
  const float inv = inv_s;
  for (int i = threadIdx.x; i < h; i += blockDim.x) y[i] = f2bf(__fmul_rn(__fmul_rn(s_sm[i], inv), bf2f(gamma[i])));
}

__global__ void silu_mul_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ u, int64_t n,
                                uint16_t* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float gf = bf2f(g[i]);
    float act = bf2f(f2bf(__fdiv_rn(gf, __fadd_rn(1.0f, spark_exp(-gf)))));
    out[i] = f2bf(__fmul_rn(act, bf2f(u[i])));
  }
}

__global__ void rope_neox_kernel(uint16_t* x, int nh, int dim, const uint16_t* __restrict__ cos_sin,
                                 const int64_t* __restrict__ pos) {
  pdl_launch_dependents();
  pdl_wait();
  const int half = dim >> 1;
  const uint16_t* cs = cos_sin + (size_t)pos[0] * dim;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < nh * half; idx += gridDim.x * blockDim.x) {
    int h = idx / half, i = idx - h * half;
    uint16_t* v = x + (size_t)h * dim;
    float a = bf2f(v[i]), b = bf2f(v[i + half]);
    float c = bf2f(cs[i]), s = bf2f(cs[i + half]);
    v[i] = f2bf(__fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)));
    v[i + half] = f2bf(__fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s)));
  }
}

// ------------------------------------------------------------------ prefill rows
// add + RMSNorm of n rows (one CTA of 256 threads per row): res_out = bf16(a + b),
// y = bf16((a + b) * rsqrt(mean((a + b)^2) + eps) * gamma).  Prefill only: the sum of
// squares is a block tree, not the decode path's canonical lane order.
__global__ void __launch_bounds__(256) add_rmsnorm_rows_kernel(const uint16_t* __restrict__ a,
                                                               const uint16_t* __restrict__ b,
                                                               const uint16_t* __restrict__ gamma, float eps,
                                                               float inv_h, int h, uint16_t* res_out, uint16_t* y) {
  extern __shared__ float s_row[];  // [h] then [8] warp partials
  const size_t off = (size_t)blockIdx.x * h;
  float part = 0.0f;
  for (int i = threadIdx.x; i < h; i += blockDim.x) {
    const float s = b ? __fadd_rn(bf2f(a[off + i]), bf2f(b[off + i])) : bf2f(a[off + i]);
    s_row[i] = s;
    if (res_out) res_out[off + i] = f2bf(s);
    part = __fmaf_rn(s, s, part);
  }
  part = butterfly_sum<32>(part);
  float* red = s_row + h;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
  __syncthreads();
  float tot = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) tot += red[w];
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(tot, inv_h), eps));
  for (int i = threadIdx.x; i < h; i += blockDim.x)
    y[off + i] = f2bf(__fmul_rn(__fmul_rn(s_row[i], inv), bf2f(gamma[i])));
}

// In-place neox RoPE of n rows of `nh` heads (row r at x + r * row_stride, position
// pos0 + r), pairs (i, i + rot/2) with cos_sin rows of rot entries (the decode kernels'
// arithmetic: separate products, then the rounded difference / sum).
__global__ void rope_rows_kernel(uint16_t* x, int64_t row_stride, int n, int nh, int dim, int rot,
                                 const uint16_t* __restrict__ cos_sin, int64_t pos0) {
  const int half = rot >> 1;
  const int64_t total = (int64_t)n * nh * half;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / (nh * half);
    const int rem = (int)(idx - r * nh * half), h = rem / half, i = rem - h * half;
    uint16_t* v = x + r * row_stride + (int64_t)h * dim;
    const uint16_t* cs = cos_sin + (pos0 + r) * rot;
    const float a = bf2f(v[i]), b = bf2f(v[i + half]);
    const float c = bf2f(cs[i]), s = bf2f(cs[i + half]);
    v[i] = f2bf(__fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)));
    v[i + half] = f2bf(__fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s)));
  }
}

// Activation * mul of n rows of a fused gate / up output gu [n][2 I] (gate columns
// [0, I), up [I, 2 I)): out [n][I] = bf16(act(bf16 gate) * bf16 up), act = the decode
// epilogues' bf16(silu) (table == nullptr) or the GELU table lookup (SparkStage.table).
__global__ void act_mul_rows_kernel(const uint16_t* __restrict__ gu, int64_t n, int inter,
                                    const uint16_t* __restrict__ table, uint16_t* __restrict__ out) {
  const int64_t total = n * inter;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / inter;
    const int i = (int)(idx - r * inter);
    const uint16_t gb = gu[r * 2 * inter + i];
    const float uf = bf2f(gu[r * 2 * inter + inter + i]);
    float act;
    if (table) {
      act = bf2f(spark_gelu_bf16(gb, table));
    } else {
      const float gf = bf2f(gb);
      act = bf2f(f2bf(__fdiv_rn(gf, __fadd_rn(1.0f, spark_exp(-gf)))));
    }
    out[idx] = f2bf(__fmul_rn(act, uf));
  }
}

// ------------------------------------------------------------------ 16-byte forms of the row kernels
// The same per-element arithmetic as the three kernels above (RMSNorm: per-thread fma
// partials, warp butterflies, the 8 warp totals in order), moved 8 bf16 values per
// 16-byte load / store.  The host uses them when the row lengths are multiples of 8 and
// the rows 16-byte aligned.
__device__ __forceinline__ void unpack8_bf16(const uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int t = 0; t < 4; t++) {
    v[2 * t] = bf_lo(w[t]);
    v[2 * t + 1] = bf_hi(w[t]);
  }
}
__device__ __forceinline__ uint4 pack8_bf16(const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int t = 0; t < 4; t++) w[t] = (uint32_t)f2bf(v[2 * t]) | ((uint32_t)f2bf(v[2 * t + 1]) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

constexpr int kRowGroupsPerThread = 4;  // add + RMSNorm: hidden <= 256 x 8 x 4 = 8192

__global__ void __launch_bounds__(256) add_rmsnorm_rows_v8_kernel(const uint16_t* __restrict__ a,
                                                                  const uint16_t* __restrict__ b,
                                                                  const uint16_t* __restrict__ gamma, float eps,
                                                                  float inv_h, int h, uint16_t* res_out, uint16_t* y) {
  __shared__ float red[8];
  const size_t off = (size_t)blockIdx.x * h;
  const int ng = h >> 3;
  float sv[kRowGroupsPerThread][8];
  float part = 0.0f;
#pragma unroll
  for (int q = 0; q < kRowGroupsPerThread; q++) {
    const int gi = threadIdx.x + q * 256;
    if (gi < ng) {
      unpack8_bf16(*reinterpret_cast<const uint4*>(a + off + 8 * gi), sv[q]);
      if (b) {
        float bv[8];
        unpack8_bf16(*reinterpret_cast<const uint4*>(b + off + 8 * gi), bv);
#pragma unroll
        for (int j = 0; j < 8; j++) sv[q][j] = __fadd_rn(sv[q][j], bv[j]);
      }
      if (res_out) *reinterpret_cast<uint4*>(res_out + off + 8 * gi) = pack8_bf16(sv[q]);
#pragma unroll
      for (int j = 0; j < 8; j++) part = __fmaf_rn(sv[q][j], sv[q][j], part);
    }
  }
  part = butterfly_sum<32>(part);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
  __syncthreads();
  float tot = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) tot += red[w];
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(tot, inv_h), eps));
#pragma unroll
  for (int q = 0; q < kRowGroupsPerThread; q++) {
    const int gi = threadIdx.x + q * 256;
    if (gi < ng) {
      float gv[8], o[8];
      unpack8_bf16(*reinterpret_cast<const uint4*>(gamma + 8 * gi), gv);
#pragma unroll
      for (int j = 0; j < 8; j++) o[j] = __fmul_rn(__fmul_rn(sv[q][j], inv), gv[j]);
      *reinterpret_cast<uint4*>(y + off + 8 * gi) = pack8_bf16(o);
    }
  }
}

// pairs (i .. i + 7, i + half .. i + half + 7) of one head of one row per thread
__global__ void rope_rows_v8_kernel(uint16_t* x, int64_t row_stride, int n, int nh, int dim, int rot,
                                    const uint16_t* __restrict__ cos_sin, int64_t pos0) {
  const int half = rot >> 1, hg = half >> 3;
  const int64_t total = (int64_t)n * nh * hg;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = idx / (nh * hg);
    const int rem = (int)(idx - r * nh * hg), h = rem / hg, i = 8 * (rem - h * hg);
    uint16_t* v = x + r * row_stride + (int64_t)h * dim;
    const uint16_t* cs = cos_sin + (pos0 + r) * rot;
    float a[8], b[8], c[8], sn[8], o0[8], o1[8];
    unpack8_bf16(*reinterpret_cast<const uint4*>(v + i), a);
    unpack8_bf16(*reinterpret_cast<const uint4*>(v + i + half), b);
    unpack8_bf16(*reinterpret_cast<const uint4*>(cs + i), c);
    unpack8_bf16(*reinterpret_cast<const uint4*>(cs + i + half), sn);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      o0[j] = __fsub_rn(__fmul_rn(a[j], c[j]), __fmul_rn(b[j], sn[j]));
      o1[j] = __fadd_rn(__fmul_rn(b[j], c[j]), __fmul_rn(a[j], sn[j]));
    }
    *reinterpret_cast<uint4*>(v + i) = pack8_bf16(o0);
    *reinterpret_cast<uint4*>(v + i + half) = pack8_bf16(o1);
  }
}

// 8 consecutive intermediate columns of one row per thread: row blockIdx.y
__global__ void act_mul_rows_v8_kernel(const uint16_t* __restrict__ gu, int inter, const uint16_t* __restrict__ table,
                                       uint16_t* __restrict__ out) {
  const int gi = blockIdx.x * blockDim.x + threadIdx.x;
  if (gi >= (inter >> 3)) return;
  const int64_t r = blockIdx.y;
  const int i = 8 * gi;
  const uint4 gw = *reinterpret_cast<const uint4*>(gu + r * 2 * inter + i);
  float uf[8], o[8];
  unpack8_bf16(*reinterpret_cast<const uint4*>(gu + r * 2 * inter + inter + i), uf);
  const uint32_t g2[4] = {gw.x, gw.y, gw.z, gw.w};
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const uint16_t gb = (uint16_t)((j & 1) ? (g2[j >> 1] >> 16) : (g2[j >> 1] & 0xffffu));
    float act;
    if (table) {
      act = bf2f(spark_gelu_bf16(gb, table));
    } else {
      const float gf = bf2f(gb);
      act = bf2f(f2bf(__fdiv_rn(gf, __fadd_rn(1.0f, spark_exp(-gf)))));
    }
    o[j] = __fmul_rn(act, uf[j]);
  }
  *reinterpret_cast<uint4*>(out + r * inter + i) = pack8_bf16(o);
}

// ------------------------------------------------------------------ slot mapping (integration/slot_mapping.py:8-22)
__global__ void slot_mapping_kernel(int64_t n, int64_t max_tokens, const int32_t* __restrict__ query_start,
                                    const int64_t* __restrict__ positions, const int32_t* __restrict__ table,
                                    int64_t bs, int64_t* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t start = query_start[0], end = query_start[1];
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < max_tokens; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t v = -1;
    if (i < n && i >= start && i < end) {
      int64_t p = positions[i], blk = p / bs;
      v = (int64_t)table[blk] * bs + (p - blk * bs);
    }
    out[i] = v;
  }
}

// ------------------------------------------------------------------ KV store
// k / v bf16 [tokens][nkv][D] -> caches [blocks][nkv][bs][D] at slot_mapping[t]
// (slot = block * bs + offset; negative slots are padding and skipped).  One thread
// moves 16 bytes.
__global__ void kv_store_kernel(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                                const int64_t* __restrict__ slots, int64_t tokens, int nkv, int D, int64_t bs,
                                uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache) {
  pdl_launch_dependents();
  pdl_wait();
  const int per_tok = nkv * D / 8;  // 16-byte pieces per token per tensor
  const int64_t total = tokens * per_tok * 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int side = (int)(i / (tokens * per_tok));
    const int64_t r = i - side * tokens * per_tok;
    const int64_t t = r / per_tok;
    const int piece = (int)(r - t * per_tok);
    const int64_t slot = slots[t];
    if (slot < 0) continue;
    const int h = piece / (D / 8), e = (piece - h * (D / 8)) * 8;
    const int64_t blk = slot / bs, off = slot - blk * bs;
    const uint16_t* src = (side ? v : k) + (t * nkv + h) * D + e;
    uint16_t* dst = (side ? v_cache : k_cache) + ((blk * nkv + h) * bs + off) * D + e;
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  }
}

// ------------------------------------------------------------------ decode bookkeeping
// The next step's kernels start only after this one has written the new token and
// position: the attention kernel reads the position before its own PDL wait, so
// the trigger comes last (after the head kernel completed, which by the chain of
// waits means the whole previous step completed).
__global__ void decode_finalize_kernel(unsigned long long* key, int32_t* token_out, int32_t* token_log,
                                       int32_t* step, int64_t* pos) {
  pdl_wait();
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    unsigned long long k = *key;
    int32_t tok = (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
    token_out[0] = tok;
    if (token_log) token_log[step ? step[0] : 0] = tok;
    *key = 0ull;
    if (pos) pos[0] += 1;
    if (step) step[0] += 1;
    __threadfence();
  }
  __syncthreads();
  pdl_launch_dependents();
}

}  // namespace spark
