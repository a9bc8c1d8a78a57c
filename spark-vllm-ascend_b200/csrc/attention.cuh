// attention.cuh -- split-KV paged GQA decode attention + log-sum-exp combine (sm_100a).
//
// Reference: kernels/attention.py:59-117 (softmax / accumulate / finish of one
// (part, kv-head) task: fp32 scores scaled after the dot product, running max,
// exp, fp32 sum, P rounded to bf16 for P.V, out = acc / l, lse = log l + m) and
// kernels/vector.py:154-192 (merge_attention: softmax over the split lse values,
// weights divided by their sum first, acc += w * O, bf16 round).
//
// KV cache layout (per layer): bf16 [num_blocks][num_kv_heads][block_size][head_dim]
// so the page of one (block, kv head) is block_size * head_dim * 2 contiguous bytes.
// Token t of the sequence lives in physical block table[t / block_size], row
// t % block_size.
//
// One CTA per (split, kv head); a split covers T = roundup16(ceil(L / S)) tokens.
// Phase 1: each lane owns one token, streams its K row (16 x 128-bit loads) and
//   forms the dot products with the G = 4 query heads of the group in fp32
//   (even dims in .x, odd dims in .y of a packed f32x2 accumulator, ascending).
// Phase 2: warp g reduces head g: max, p = exp(score - max), l = 32-lane sum
//   (token i into lane i mod 32, ascending, xor butterfly), P rounded to bf16.
// Phase 3: thread (g, dim pair) accumulates P.V over the split's tokens in
//   ascending order from a cp.async-staged V ring in shared memory.
#pragma once

#include "common.cuh"

namespace spark {

constexpr int kAttnThreads = 256;
constexpr int kAttnChunk = 64;     // tokens per V stage
constexpr int kAttnStages = 4;     // V ring depth
constexpr int kAttnMaxSplitTokens = 2048;

struct AttnArgs {
  const uint16_t* q;          // bf16 [nq][D]
  const uint16_t* k_cache;    // bf16 [blocks][nkv][bs][D]
  const uint16_t* v_cache;
  const int32_t* block_table; // int32 [max_blocks]
  const int64_t* pos64;       // sequence length = pos + 1 (one of pos64 / pos32 / seq_len32)
  const int32_t* pos32;
  const int32_t* seq_len32;
  int nq, nkv, block_size, splits, t_alloc;
  float scale;
  float* part_o;              // fp32 [splits][nq][D]
  float* part_lse;            // fp32 [splits][nq]
  int* error;                 // set to 1 when the split is longer than t_alloc
};

__device__ __forceinline__ int64_t attn_seq_len(const AttnArgs& a) {
  if (a.seq_len32) return a.seq_len32[0];
  if (a.pos64) return a.pos64[0] + 1;
  return (int64_t)a.pos32[0] + 1;
}

__device__ __forceinline__ int64_t attn_split_tokens(int64_t len, int splits) {
  int64_t t = (len + splits - 1) / splits;
  return (t + 15) / 16 * 16;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int D, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_split_kernel(const AttnArgs a) {
  static_assert(D == 128 && G == 4, "this kernel is specialised for head_dim 128, 4 query heads per kv head");
  extern __shared__ __align__(16) float smem[];
  float* qf = smem;                                   // [G][D]
  float* scores = qf + G * D;                         // [G][t_alloc]
  float* stat = scores + (size_t)G * a.t_alloc;       // [G][2]: l, m
  uint16_t* vring = reinterpret_cast<uint16_t*>(stat + 2 * G + 8);  // [stages][chunk][D]

  pdl_launch_dependents();
  pdl_wait();

  const int s = blockIdx.x, hk = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int64_t len = attn_seq_len(a);
  const int64_t T = attn_split_tokens(len, a.splits);
  const int64_t t0 = (int64_t)s * T;
  const int n = (int)((len - t0) < T ? (len - t0) : T);
  const size_t head_stride = (size_t)a.block_size * D;
  const size_t block_stride = (size_t)a.nkv * head_stride;

  if (n <= 0 || T > a.t_alloc) {
    if (T > a.t_alloc && tid == 0 && a.error) atomicExch(a.error, 1);
    for (int i = tid; i < G * D; i += kAttnThreads) {
      int g = i / D, dd = i - g * D;
      a.part_o[((size_t)s * a.nq + hk * G + g) * D + dd] = 0.0f;
    }
    if (tid < G) a.part_lse[(size_t)s * a.nq + hk * G + tid] = __int_as_float(0xff800000);
    return;
  }

  // q of the group -> fp32
  for (int i = tid; i < G * D; i += kAttnThreads) qf[i] = bf2f(a.q[(size_t)(hk * G) * D + i]);

  // V ring prefetch of the first stages
  const int nchunks = (n + kAttnChunk - 1) / kAttnChunk;
  auto issue_v = [&](int c) {
    if (c < nchunks) {
      uint16_t* dst = vring + (size_t)(c % kAttnStages) * kAttnChunk * D;
#pragma unroll
      for (int m = 0; m < (kAttnChunk * D * 2 / 16) / kAttnThreads; m++) {
        int idx = tid + m * kAttnThreads;      // 16-byte piece
        int j = idx / (D * 2 / 16), piece = idx % (D * 2 / 16);
        int i = c * kAttnChunk + j;
        if (i < n) {
          int64_t t = t0 + i;
          int64_t blk = a.block_table[t / a.block_size], off = t % a.block_size;
          const uint16_t* src = a.v_cache + blk * block_stride + hk * head_stride + off * D + piece * 8;
          cp_async16(dst + (size_t)j * D + piece * 8, src);
        }
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int c = 0; c < kAttnStages - 1; c++) issue_v(c);
  __syncthreads();

  // phase 1: scores
  for (int i = tid; i < n; i += kAttnThreads) {
    int64_t t = t0 + i;
    int64_t blk = a.block_table[t / a.block_size], off = t % a.block_size;
    const uint4* kr = reinterpret_cast<const uint4*>(a.k_cache + blk * block_stride + hk * head_stride + off * D);
    uint4 kv[D / 8];
#pragma unroll
    for (int c = 0; c < D / 8; c++) kv[c] = ldg_stream(kr + c);
    float2 acc[G];
#pragma unroll
    for (int g = 0; g < G; g++) acc[g] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int c = 0; c < D / 8; c++) {
      const uint32_t w4[4] = {kv[c].x, kv[c].y, kv[c].z, kv[c].w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float2 kk = make_float2(bf_lo(w4[e]), bf_hi(w4[e]));
        const int dd = c * 8 + e * 2;
#pragma unroll
        for (int g = 0; g < G; g++) {
          const float2 qq = *reinterpret_cast<const float2*>(qf + g * D + dd);
          acc[g] = __ffma2_rn(qq, kk, acc[g]);
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; g++) scores[(size_t)g * a.t_alloc + i] = __fmul_rn(__fadd_rn(acc[g].x, acc[g].y), a.scale);
  }
  __syncthreads();

  // phase 2: softmax statistics, warp g handles head g
  if (warp < G) {
    float* sc = scores + (size_t)warp * a.t_alloc;
    float m = __int_as_float(0xff800000);
    for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[i]);
    m = warp_max(m);
    float l = 0.0f;
    for (int i = lane; i < n; i += 32) {
      float p = spark_exp(__fsub_rn(sc[i], m));
      l = __fadd_rn(l, p);
      sc[i] = bf2f(f2bf(p));
    }
    l = butterfly_sum<32>(l);
    if (lane == 0) {
      stat[warp * 2 + 0] = l;
      stat[warp * 2 + 1] = m;
    }
  }

  // phase 3: P.V
  const int g = tid / (D / 2), dp = tid % (D / 2);
  const float* pg = scores + (size_t)g * a.t_alloc;
  float2 o = make_float2(0.0f, 0.0f);
  for (int c = 0; c < nchunks; c++) {
    __syncthreads();  // stage (c-1) % stages fully consumed; phase 2 done on first pass
    issue_v(c + kAttnStages - 1);
    cp_async_wait<kAttnStages - 1>();
    __syncthreads();
    const uint16_t* vs = vring + (size_t)(c % kAttnStages) * kAttnChunk * D;
    const int jn = (n - c * kAttnChunk) < kAttnChunk ? (n - c * kAttnChunk) : kAttnChunk;
    for (int j = 0; j < jn; j++) {
      const uint32_t vw = *reinterpret_cast<const uint32_t*>(vs + (size_t)j * D + 2 * dp);
      const float p = pg[c * kAttnChunk + j];
      o = __ffma2_rn(make_float2(p, p), make_float2(bf_lo(vw), bf_hi(vw)), o);
    }
  }
  cp_async_wait<0>();
  const float l = stat[g * 2 + 0], m = stat[g * 2 + 1];
  const int hq = hk * G + g;
  float2 out = make_float2(__fdiv_rn(o.x, l), __fdiv_rn(o.y, l));
  *reinterpret_cast<float2*>(a.part_o + ((size_t)s * a.nq + hq) * D + 2 * dp) = out;
  if (dp == 0) a.part_lse[(size_t)s * a.nq + hq] = __fadd_rn(spark_log(l), m);
}

// ------------------------------------------------------------------ combine
struct CombineArgs {
  const float* part_o;    // fp32 [splits][nq][D]
  const float* part_lse;  // fp32 [splits][nq]
  int splits, nq, dim;
  uint16_t* out;          // bf16 [nq][D]
};

// One CTA per query head, one thread per output dim.
__global__ void __launch_bounds__(128) attn_combine_kernel(const CombineArgs a) {
  extern __shared__ float wsm[];  // [splits]
  __shared__ float mx_s;
  pdl_launch_dependents();
  pdl_wait();
  const int hq = blockIdx.x;
  if (threadIdx.x == 0) {
    float mx = __int_as_float(0xff800000);
    for (int s = 0; s < a.splits; s++) mx = fmaxf(mx, a.part_lse[(size_t)s * a.nq + hq]);
    float den = 0.0f;
    if (mx != __int_as_float(0xff800000)) {
      for (int s = 0; s < a.splits; s++) {
        float v = a.part_lse[(size_t)s * a.nq + hq];
        float w = (v == __int_as_float(0xff800000)) ? 0.0f : spark_exp(__fsub_rn(v, mx));
        wsm[s] = w;
        den = __fadd_rn(den, w);
      }
      for (int s = 0; s < a.splits; s++) wsm[s] = __fdiv_rn(wsm[s], den);
    }
    mx_s = mx;
  }
  __syncthreads();
  const bool all_empty = mx_s == __int_as_float(0xff800000);
  for (int dd = threadIdx.x; dd < a.dim; dd += blockDim.x) {
    float acc = 0.0f;
    if (!all_empty) {
      for (int s = 0; s < a.splits; s++) {
        if (a.part_lse[(size_t)s * a.nq + hq] == __int_as_float(0xff800000)) continue;
        acc = __fadd_rn(acc, __fmul_rn(wsm[s], a.part_o[((size_t)s * a.nq + hq) * a.dim + dd]));
      }
    }
    a.out[(size_t)hq * a.dim + dd] = f2bf(acc);
  }
}

}  // namespace spark
