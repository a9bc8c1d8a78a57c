// attention.cuh -- split-KV paged GQA decode attention + log-sum-exp combine (sm_100a).
//
// Reference: kernels/attention.py:59-117 (softmax / accumulate / finish of one
// (part, kv-head) task: fp32 scores scaled after the dot product, running max,
// exp, fp32 sum, P rounded to bf16 for P.V, out = acc / l, lse = log l + m) and
// kernels/vector.py:46-83 (merge_attention: softmax over the split lse values,
// weights divided by their sum first, acc += w * O, bf16 round).
//
// KV cache layout (per layer): bf16 [num_blocks][num_kv_heads][block_size][head_dim]
// so the page of one (block, kv head) is block_size * head_dim * 2 contiguous bytes.
// Token t of the sequence lives in physical block table[t / block_size], row
// t % block_size.
//
// One CTA (128 threads) per (split, kv head); a split covers T = roundup16(ceil(L / S))
// tokens, processed in chunks of 128.
// Fetch: K and V rows are copied with cp.async into shared memory (K rows padded
//   to 272 bytes); rows older than the current position are requested before the
//   programmatic-launch wait, the current token's row (written by the preceding
//   QKV kernel) after it.
// Scores: 8 lanes per token; lane j owns dims 8j..8j+7 and 64+8j..64+8j+7, holds
//   q for two query heads in registers, accumulates the even / odd positions of
//   its dims in the .x / .y halves of a packed f32x2 FMA, and the 8 lane values
//   are combined by an xor butterfly (4, 2, 1); score = sum * scale.
// Softmax: warp g reduces head g: max, p = exp(score - max), l = 32-lane sum
//   (token i into lane i mod 32, ascending, xor butterfly), P rounded to bf16.
// P.V: thread (head pair, dim pair) accumulates over the tokens in ascending order.
// Combine (optional, fused): after writing its partial, each CTA bumps a per-kv-head
//   arrival counter; the CTA that arrives last merges the splits of its four query
//   heads in the canonical order and resets the counter for the next call.
//
// Wide form (attn_decode_wide_kernel, splits of at most kWideMaxTokens tokens): the same
// arithmetic in the same orders, laid out for bandwidth -- 16 warps per (split, kv head),
// the split's whole K and V brought into shared memory by one bulk copy per page segment
// and side (all in flight at once; K on one mbarrier, V on another, landing while the
// scores and softmax run; the block-table entries of the split come in one round trip of
// warp 0); P.V by 128 threads of (head pair, dim pair) reading each
// token's bf16 P of the pair with one broadcast load (shared-memory wavefronts, not
// arithmetic, bound that phase).
#pragma once

#include "common.cuh"
#include "q4_gemv_ring.cuh"

namespace spark {

constexpr int kAttnThreads = 128;
constexpr int kAttnChunk = 128;   // tokens per K / V chunk
constexpr int kKRowBytes = 272;   // padded K row in shared memory (conflict-free 8-lane reads)
constexpr int kVRowBytes = 256;
constexpr int kAttnMaxSplitTokens = 2048;
constexpr int kAttnMaxFusedSplits = 256;

struct AttnArgs {
  const uint16_t* q;          // bf16 [nq][D]
  const uint16_t* k_cache;    // bf16 [blocks][nkv][bs][D]
  const uint16_t* v_cache;
  const int32_t* block_table; // int32 [max_blocks]
  const int64_t* pos64;       // sequence length = pos + 1 (one of pos64 / pos32 / seq_len32)
  const int32_t* pos32;
  const int32_t* seq_len32;
  int nq, nkv, block_size, splits, t_alloc, kv_slots;
  float scale;
  float* part_o;              // fp32 [splits][nq][D]
  float* part_lse;            // fp32 [splits][nq]
  int* error;                 // set to 1 when the split is longer than t_alloc
  int* counters;              // fused combine: int [nkv], zero before the first call
  uint16_t* out;              // fused combine: bf16 [nq][D]; null = partials only
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
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Copy the rows of split-local tokens [c*128, c*128+rows) of one cache into a slot.
// skip >= 0: leave that token out; only >= 0: copy only that token.
template <int D>
__device__ __forceinline__ void attn_issue_rows(const AttnArgs& a, const uint16_t* cache, unsigned char* slot,
                                                int row_bytes, int64_t tbase, int rows, int hk, int64_t skip,
                                                int64_t only) {
  const size_t head_stride = (size_t)a.block_size * D;
  const size_t block_stride = (size_t)a.nkv * head_stride;
  constexpr int kPieces = D * 2 / 16;
  if (only >= 0) {
    const int r = (int)(only - tbase);
    if (r < 0 || r >= rows) return;
    for (int p = threadIdx.x; p < kPieces; p += blockDim.x) {
      const int64_t blk = a.block_table[only / a.block_size], off = only % a.block_size;
      cp_async16(slot + (size_t)r * row_bytes + p * 16, cache + blk * block_stride + hk * head_stride + off * D + p * 8);
    }
    return;
  }
  for (int idx = threadIdx.x; idx < rows * kPieces; idx += blockDim.x) {
    const int r = idx / kPieces, p = idx - r * kPieces;
    const int64_t t = tbase + r;
    if (t == skip) continue;
    const int64_t blk = a.block_table[t / a.block_size], off = t % a.block_size;
    cp_async16(slot + (size_t)r * row_bytes + p * 16, cache + blk * block_stride + hk * head_stride + off * D + p * 8);
  }
}

// Merge the split partials of G query heads [hq0, hq0+G) into bf16 out, in the
// canonical order of merge_attention (kernels/vector.py:46-83): M = max lse,
// w_s = exp(lse_s - M) (0 for empty splits), den = sum_s w_s in ascending s,
// w_s /= den, out = bf16(sum_s w_s * O_s) in ascending s (product, then add).
// The weights are computed in parallel, only the two canonical sums are serial;
// partials are staged through shared memory (buf, buf_bytes) with all loads in
// flight.  wn: [G][kAttnMaxFusedSplits] floats, mx: [G][2] floats.  128 threads.
// NT threads (128 or 512; warps 0..G-1 compute the weights).
template <int D, int G, int NT = 128>
__device__ __forceinline__ void attn_merge_heads(const float* part_o, const float* part_lse, int splits, int nq,
                                                 int hq0, uint16_t* out, float* wn, float* mx,
                                                 unsigned char* buf, size_t buf_bytes) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;  // warp g <-> head g (first G warps)
  const float ninf = __int_as_float(0xff800000);
  const int per_split = G * D * 4;
  const int chunk = (int)(buf_bytes / per_split) < splits ? (int)(buf_bytes / per_split) : splits;
  auto fetch = [&](int s0) {  // partials of splits s0 .. s0 + chunk - 1 into buf
    const int ns = min(chunk, splits - s0);
    for (int idx = tid; idx < ns * (G * D / 4); idx += NT) {
      const int sp = idx / (G * D / 4), p = idx - sp * (G * D / 4);
      cp_async16(buf + (size_t)sp * per_split + p * 16, part_o + ((size_t)(s0 + sp) * nq + hq0) * D + p * 4);
    }
    cp_async_commit();
  };
  fetch(0);  // the first partials travel while the weights are computed
  if (warp < G) {
  float* w = wn + warp * kAttnMaxFusedSplits;
  // lse -> weights (warp g handles head g)
  float m = ninf;
  for (int sp = lane; sp < splits; sp += 32) {
    const float v = __ldcg(part_lse + (size_t)sp * nq + hq0 + warp);
    w[sp] = v;
    m = fmaxf(m, v);
  }
  m = warp_max(m);
  __syncwarp();
  if (m != ninf)
    for (int sp = lane; sp < splits; sp += 32) w[sp] = (w[sp] == ninf) ? -1.0f : spark_exp(__fsub_rn(w[sp], m));
  __syncwarp();
  if (lane == 0) {
    float den = 0.0f;
    if (m != ninf)
      for (int sp = 0; sp < splits; sp++) den = __fadd_rn(den, w[sp] < 0.0f ? 0.0f : w[sp]);
    mx[warp * 2] = den;
    mx[warp * 2 + 1] = m;
  }
  __syncwarp();
  const float den = mx[warp * 2];
  if (m != ninf)
    for (int sp = lane; sp < splits; sp += 32) w[sp] = w[sp] < 0.0f ? -1.0f : __fdiv_rn(w[sp], den);
  }
  __syncthreads();
  // weighted sum; empty splits (w == -1) are skipped
  float acc[G * D / NT];
#pragma unroll
  for (int i = 0; i < G * D / NT; i++) acc[i] = 0.0f;
  for (int s0 = 0; s0 < splits; s0 += chunk) {
    const int ns = min(chunk, splits - s0);
    if (s0 > 0) {
      __syncthreads();  // the previous round's reads of buf
      fetch(s0);
    }
    cp_async_wait_all();
    __syncthreads();
    const float* ob = reinterpret_cast<const float*>(buf);
#pragma unroll
    for (int i = 0; i < G * D / NT; i++) {
      const int e = tid + NT * i, g = e / D;
      if (mx[g * 2 + 1] == ninf) continue;
      const float* wg = wn + g * kAttnMaxFusedSplits + s0;
      float a = acc[i];
      for (int sp = 0; sp < ns; sp++) {
        const float ww = wg[sp];
        if (ww < 0.0f) continue;
        a = __fadd_rn(a, __fmul_rn(ww, ob[(size_t)sp * (G * D) + e]));
      }
      acc[i] = a;
    }
  }
#pragma unroll
  for (int i = 0; i < G * D / NT; i++) {
    const int e = tid + NT * i;
    out[(size_t)hq0 * D + e] = f2bf(acc[i]);
  }
}

template <int D, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
  static_assert(D == 128 && G == 4, "specialised for head_dim 128, 4 query heads per kv head");
  extern __shared__ __align__(16) unsigned char smem_at[];
  float* scores = reinterpret_cast<float*>(smem_at);                       // [G][t_alloc]
  float* stat = scores + (size_t)G * a.t_alloc;                             // [G][2]: l, m
  float* wn = stat + 2 * G;                                                 // [G][kAttnMaxFusedSplits]
  int* flag = reinterpret_cast<int*>(wn + G * kAttnMaxFusedSplits);         // [4]
  unsigned char* kbuf = reinterpret_cast<unsigned char*>(flag + 4);         // [kv_slots][128][272]
  unsigned char* vbuf = kbuf + (size_t)a.kv_slots * kAttnChunk * kKRowBytes;  // [kv_slots][128][256]

  pdl_launch_dependents();

  const int s = blockIdx.x, hk = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  // Everything read before pdl_wait is stable during this step: the position and
  // block table are written before the step starts, and cache rows older than the
  // current position were written by earlier steps.
  const int64_t len = attn_seq_len(a);
  const int64_t pos = len - 1;
  const int64_t T = attn_split_tokens(len, a.splits);
  const int64_t t0 = (int64_t)s * T;
  const int n = (int)((len - t0) < T ? (len - t0) : T);
  const bool ok = n > 0 && T <= a.t_alloc;
  const int nch = ok ? (n + kAttnChunk - 1) / kAttnChunk : 0;
  const int slots = a.kv_slots;

  if (ok) {
    for (int c = 0; c < nch && c < slots; c++) {
      const int rows = min(kAttnChunk, n - c * kAttnChunk);
      attn_issue_rows<D>(a, a.k_cache, kbuf + (size_t)c * kAttnChunk * kKRowBytes, kKRowBytes, t0 + c * kAttnChunk, rows,
                         hk, pos, -1);
      attn_issue_rows<D>(a, a.v_cache, vbuf + (size_t)c * kAttnChunk * kVRowBytes, kVRowBytes, t0 + c * kAttnChunk, rows,
                         hk, pos, -1);
    }
    cp_async_commit();
  }

  pdl_wait();

  const int hq0 = hk * G;
  if (!ok) {
    if (n > 0 && tid == 0 && a.error) atomicExch(a.error, 1);
    for (int i = tid; i < G * D; i += kAttnThreads) a.part_o[((size_t)s * a.nq + hq0) * D + i] = 0.0f;
    if (tid < G) a.part_lse[(size_t)s * a.nq + hq0 + tid] = __int_as_float(0xff800000);
  } else {
    // the current token's rows, if they fall into an already requested chunk
    const int cpos = (int)((pos - t0) / kAttnChunk);
    if (pos >= t0 && pos < t0 + n && cpos < slots) {
      const int rows = min(kAttnChunk, n - cpos * kAttnChunk);
      attn_issue_rows<D>(a, a.k_cache, kbuf + (size_t)cpos * kAttnChunk * kKRowBytes, kKRowBytes,
                         t0 + cpos * kAttnChunk, rows, hk, -1, pos);
      attn_issue_rows<D>(a, a.v_cache, vbuf + (size_t)cpos * kAttnChunk * kVRowBytes, kVRowBytes,
                         t0 + cpos * kAttnChunk, rows, hk, -1, pos);
    }
    cp_async_commit();

    // q of this lane's dims for its head pair, fp32 in registers
    const int j = lane & 7, grp = lane >> 3;
    const int hp = warp >> 1, wsub = warp & 1;
    float2 qr[2][8];
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
      const uint16_t* qh = a.q + (size_t)(hq0 + 2 * hp + hh) * D;
      const uint4 q0 = *reinterpret_cast<const uint4*>(qh + 8 * j);
      const uint4 q1 = *reinterpret_cast<const uint4*>(qh + 64 + 8 * j);
      const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int m = 0; m < 8; m++) qr[hh][m] = make_float2(bf_lo(w[m]), bf_hi(w[m]));
    }
    cp_async_wait_all();
    __syncthreads();

    // ---- scores
    for (int c = 0; c < nch; c++) {
      const int slot = c % slots;
      if (c >= slots) {
        // chunk c was not prefetched: fetch it into its slot now (all earlier uses done)
        __syncthreads();
        attn_issue_rows<D>(a, a.k_cache, kbuf + (size_t)slot * kAttnChunk * kKRowBytes, kKRowBytes,
                           t0 + c * kAttnChunk, min(kAttnChunk, n - c * kAttnChunk), hk, -1, -1);
        cp_async_commit();
        cp_async_wait_all();
        __syncthreads();
      }
      const int rows = min(kAttnChunk, n - c * kAttnChunk);
      const unsigned char* kb = kbuf + (size_t)slot * kAttnChunk * kKRowBytes;
      for (int r0 = 0; r0 < rows; r0 += 8) {
        const int r = r0 + wsub * 4 + grp;
        float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
        if (r < rows) {
          const uint4 k0 = *reinterpret_cast<const uint4*>(kb + (size_t)r * kKRowBytes + 16 * j);
          const uint4 k1 = *reinterpret_cast<const uint4*>(kb + (size_t)r * kKRowBytes + 128 + 16 * j);
          const uint32_t w[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
          for (int m = 0; m < 8; m++) {
            const float2 kk = make_float2(bf_lo(w[m]), bf_hi(w[m]));
            acc0 = __ffma2_rn(qr[0][m], kk, acc0);
            acc1 = __ffma2_rn(qr[1][m], kk, acc1);
          }
        }
        float v0 = __fadd_rn(acc0.x, acc0.y), v1 = __fadd_rn(acc1.x, acc1.y);
#pragma unroll
        for (int off = 4; off >= 1; off >>= 1) {
          v0 = __fadd_rn(v0, __shfl_xor_sync(0xffffffffu, v0, off));
          v1 = __fadd_rn(v1, __shfl_xor_sync(0xffffffffu, v1, off));
        }
        if (j == 0 && r < rows) {
          const int i = c * kAttnChunk + r;
          scores[(size_t)(2 * hp) * a.t_alloc + i] = __fmul_rn(v0, a.scale);
          scores[(size_t)(2 * hp + 1) * a.t_alloc + i] = __fmul_rn(v1, a.scale);
        }
      }
    }
    __syncthreads();

    // ---- softmax statistics, warp g handles head g
    {
      float* sc = scores + (size_t)warp * a.t_alloc;
      float m = __int_as_float(0xff800000);
      for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[i]);
      m = warp_max(m);
      float l = 0.0f;
      for (int i = lane; i < n; i += 32) {
        const float p = spark_exp(__fsub_rn(sc[i], m));
        l = __fadd_rn(l, p);
        sc[i] = bf2f(f2bf(p));
      }
      l = butterfly_sum<32>(l);
      if (lane == 0) {
        stat[warp * 2 + 0] = l;
        stat[warp * 2 + 1] = m;
      }
    }
    __syncthreads();

    // ---- P.V: thread (head pair, dim pair)
    const int php = tid >> 6, dp = tid & 63;
    const float* p0 = scores + (size_t)(2 * php) * a.t_alloc;
    const float* p1 = scores + (size_t)(2 * php + 1) * a.t_alloc;
    float2 o0 = make_float2(0.0f, 0.0f), o1 = make_float2(0.0f, 0.0f);
    for (int c = 0; c < nch; c++) {
      const int slot = c % slots;
      if (c >= slots) {
        __syncthreads();
        attn_issue_rows<D>(a, a.v_cache, vbuf + (size_t)slot * kAttnChunk * kVRowBytes, kVRowBytes,
                           t0 + c * kAttnChunk, min(kAttnChunk, n - c * kAttnChunk), hk, -1, -1);
        cp_async_commit();
        cp_async_wait_all();
        __syncthreads();
      }
      const int rows = min(kAttnChunk, n - c * kAttnChunk);
      const unsigned char* vb = vbuf + (size_t)slot * kAttnChunk * kVRowBytes + 4 * dp;
      const int ib = c * kAttnChunk;
#pragma unroll 4
      for (int r = 0; r < rows; r++) {
        const uint32_t vw = *reinterpret_cast<const uint32_t*>(vb + (size_t)r * kVRowBytes);
        const float2 vv = make_float2(bf_lo(vw), bf_hi(vw));
        const float pa = p0[ib + r], pb = p1[ib + r];
        o0 = __ffma2_rn(make_float2(pa, pa), vv, o0);
        o1 = __ffma2_rn(make_float2(pb, pb), vv, o1);
      }
    }
    const int ha = 2 * php, hb = 2 * php + 1;
    const float la = stat[ha * 2], lb = stat[hb * 2];
    *reinterpret_cast<float2*>(a.part_o + ((size_t)s * a.nq + hq0 + ha) * D + 2 * dp) =
        make_float2(__fdiv_rn(o0.x, la), __fdiv_rn(o0.y, la));
    *reinterpret_cast<float2*>(a.part_o + ((size_t)s * a.nq + hq0 + hb) * D + 2 * dp) =
        make_float2(__fdiv_rn(o1.x, lb), __fdiv_rn(o1.y, lb));
    if (dp == 0) {
      a.part_lse[(size_t)s * a.nq + hq0 + ha] = __fadd_rn(spark_log(la), stat[ha * 2 + 1]);
      a.part_lse[(size_t)s * a.nq + hq0 + hb] = __fadd_rn(spark_log(lb), stat[hb * 2 + 1]);
    }
  }

  if (a.out == nullptr) return;
  // ---- fused combine: the last split CTA of this kv head merges its four q heads
  __threadfence();
  __syncthreads();
  if (tid == 0) flag[0] = (atomicAdd(&a.counters[hk], 1) == a.splits - 1);
  __syncthreads();
  if (!flag[0]) return;
  __threadfence();
  attn_merge_heads<D, G>(a.part_o, a.part_lse, a.splits, a.nq, hq0, a.out, wn, stat, kbuf,
                         (size_t)a.kv_slots * kAttnChunk * (kKRowBytes + kVRowBytes));
  if (tid == 0) a.counters[hk] = 0;
}


// ------------------------------------------------------------------ wide kernel
constexpr int kWideThreads = 512;
constexpr int kWideMaxTokens = 400;  // K + V of the split (2 x 256 B per token) stay in shared memory
constexpr int kWideMaxSegs = 8;      // page segments of a split (block_size >= 64)

// Shared memory of the wide kernel for splits of t_alloc tokens.
__host__ __device__ constexpr size_t attn_wide_smem(int t_alloc) {
  return (size_t)t_alloc * 512 + (size_t)(8 * t_alloc + 8 + 4 * kAttnMaxFusedSplits) * 4 + 16 + 16;
}

template <int D, int G>
__global__ void __launch_bounds__(kWideThreads, 1) attn_decode_wide_kernel(const AttnArgs a) {
  static_assert(D == 128 && G == 4, "specialised for head_dim 128, 4 query heads per kv head");
  extern __shared__ __align__(128) unsigned char smem_w[];
  const int TA = a.t_alloc;
  unsigned char* kbuf = smem_w;                                             // [TA][256]
  unsigned char* vbuf = kbuf + (size_t)TA * (2 * D);                        // [TA][256]
  float* scores = reinterpret_cast<float*>(vbuf + (size_t)TA * (2 * D));   // [G][TA]
  float* p4 = scores + (size_t)G * TA;                                      // [TA][G]: bf16 P as fp32
  float* stat = p4 + (size_t)G * TA;                                        // [G][2]: l, m
  float* wn = stat + 2 * G;                                                 // [G][kAttnMaxFusedSplits]
  int* flag = reinterpret_cast<int*>(wn + G * kAttnMaxFusedSplits);         // [4]
  unsigned long long* bars = reinterpret_cast<unsigned long long*>(flag + 4);  // K, V

  pdl_launch_dependents();

  const int s = blockIdx.x, hk = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int64_t len = attn_seq_len(a);
  const int64_t pos = len - 1;
  const int64_t T = attn_split_tokens(len, a.splits);
  const int64_t t0 = (int64_t)s * T;
  const int n = (int)((len - t0) < T ? (len - t0) : T);
  const int bs = a.block_size;
  const int64_t pg0 = t0 / bs;  // the split's first page
  const int nseg = n > 0 ? (int)((t0 + n - 1) / bs - pg0 + 1) : 0;
  bool ok = n > 0 && T <= a.t_alloc && nseg <= kWideMaxSegs;
  const uint32_t kbar = smem_u32(bars), vbar = kbar + 8;
  const size_t head_stride = (size_t)bs * D, block_stride = (size_t)a.nkv * head_stride;
  // the decoded token (pos, the last token of the last split) is written by the preceding
  // QKV kernel: its rows are copied after the programmatic-launch wait, older rows before
  const bool has_pos = ok && pos < t0 + n;
  int64_t pos_blk = 0;  // (warp 0) page of the decoded token
  if (ok && warp == 0) {
    const int64_t my_blk = lane < nseg ? (int64_t)a.block_table[pg0 + lane] : 0;  // one round trip
    if (lane == 0) {
      mbar_init(kbar, 1);
      mbar_init(vbar, 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      mbar_expect_tx(kbar, (uint32_t)n * (2 * D));
      mbar_expect_tx(vbar, (uint32_t)n * (2 * D));
    }
    // segment g: the split's tokens in page pg0 + g; K of every segment, then V
    for (int side = 0; side < 2; side++) {
      const uint16_t* cache = side ? a.v_cache : a.k_cache;
      unsigned char* dst = side ? vbuf : kbuf;
      for (int g = 0; g < nseg; g++) {
        const int64_t blk = __shfl_sync(0xffffffffu, my_blk, g);
        if (g == nseg - 1) pos_blk = blk;
        if (lane == 0) {
          const int64_t ta = (pg0 + g) * bs > t0 ? (pg0 + g) * bs : t0;
          const int64_t tb = (pg0 + g + 1) * bs < t0 + n ? (pg0 + g + 1) * bs : t0 + n;
          const int rows = (int)(tb - ta);
          const int pre = (has_pos && g == nseg - 1) ? rows - 1 : rows;  // the decoded row comes later
          if (pre > 0)
            bulk_g2s(smem_u32(dst + (size_t)(ta - t0) * (2 * D)),
                     cache + blk * block_stride + hk * head_stride + (size_t)(ta - (pg0 + g) * bs) * D,
                     (uint32_t)pre * (2 * D), side ? vbar : kbar);
        }
      }
    }
  }
  __syncthreads();  // the barriers are initialised before any thread polls them
  pdl_wait();
  if (has_pos && tid == 0) {  // the decoded token's rows (pos = t0 + n - 1)
    const size_t src = pos_blk * block_stride + hk * head_stride + (size_t)(pos % bs) * D;
    bulk_g2s(smem_u32(kbuf + (size_t)(n - 1) * (2 * D)), a.k_cache + src, 2 * D, kbar);
    bulk_g2s(smem_u32(vbuf + (size_t)(n - 1) * (2 * D)), a.v_cache + src, 2 * D, vbar);
  }
  const int hq0 = hk * G;
  const float ninf = __int_as_float(0xff800000);
  bool landed = true;
  if (ok) {
    // q of this lane's dims for the 4 heads, fp32 in registers
    const int j = lane & 7, grp = lane >> 3;
    float2 qr[G][8];
#pragma unroll
    for (int hh = 0; hh < G; hh++) {
      const uint16_t* qh = a.q + (size_t)(hq0 + hh) * D;
      const uint4 q0 = *reinterpret_cast<const uint4*>(qh + 8 * j);
      const uint4 q1 = *reinterpret_cast<const uint4*>(qh + 64 + 8 * j);
      const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int m = 0; m < 8; m++) qr[hh][m] = make_float2(bf_lo(w[m]), bf_hi(w[m]));
    }
    landed = __syncthreads_and(mbar_wait(kbar, 0)) != 0;
    if (landed) {
      // ---- scores: warp w takes tokens 4 (w + 16 i) + grp; per token and head the 8-lane
      // order of the narrow kernel
      for (int i0 = warp * 4; i0 < n; i0 += (kWideThreads / 32) * 4) {
        const int r = i0 + grp;
        float2 acc[G];
#pragma unroll
        for (int hh = 0; hh < G; hh++) acc[hh] = make_float2(0.0f, 0.0f);
        if (r < n) {
          const uint4 k0 = *reinterpret_cast<const uint4*>(kbuf + (size_t)r * (2 * D) + 16 * j);
          const uint4 k1 = *reinterpret_cast<const uint4*>(kbuf + (size_t)r * (2 * D) + 128 + 16 * j);
          const uint32_t w[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
          for (int m = 0; m < 8; m++) {
            const float2 kk = make_float2(bf_lo(w[m]), bf_hi(w[m]));
#pragma unroll
            for (int hh = 0; hh < G; hh++) acc[hh] = __ffma2_rn(qr[hh][m], kk, acc[hh]);
          }
        }
#pragma unroll
        for (int hh = 0; hh < G; hh++) {
          float v = __fadd_rn(acc[hh].x, acc[hh].y);
#pragma unroll
          for (int off = 4; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
          if (j == 0 && r < n) scores[(size_t)hh * TA + r] = __fmul_rn(v, a.scale);
        }
      }
      __syncthreads();
      // ---- softmax statistics, warp g handles head g
      if (warp < G) {
        float* sc = scores + (size_t)warp * TA;
        float m = ninf;
        for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[i]);
        m = warp_max(m);
        float l = 0.0f;
        for (int i = lane; i < n; i += 32) {
          const float p = spark_exp(__fsub_rn(sc[i], m));
          l = __fadd_rn(l, p);
          p4[(size_t)i * G + warp] = bf2f(f2bf(p));
        }
        l = butterfly_sum<32>(l);
        if (lane == 0) {
          stat[warp * 2 + 0] = l;
          stat[warp * 2 + 1] = m;
        }
      }
      landed = __syncthreads_and(mbar_wait(vbar, 0)) != 0;
    }
    if (landed) {
      // ---- P.V: thread (head pair hp, dim pair dp) of the first 128, tokens ascending
      if (tid < 128) {
        const int hp = tid >> 6, dp = tid & 63;
        const float* pp = p4 + 2 * hp;
        const unsigned char* vb = vbuf + 4 * dp;
        float2 o0 = make_float2(0.0f, 0.0f), o1 = make_float2(0.0f, 0.0f);
        int r = 0;
        for (; r + 8 <= n; r += 8) {
          uint32_t vw[8];
          float2 pw[8];
#pragma unroll
          for (int q = 0; q < 8; q++) {
            vw[q] = *reinterpret_cast<const uint32_t*>(vb + (size_t)(r + q) * (2 * D));
            pw[q] = *reinterpret_cast<const float2*>(pp + (size_t)(r + q) * G);
          }
#pragma unroll
          for (int q = 0; q < 8; q++) {
            const float2 vv = make_float2(bf_lo(vw[q]), bf_hi(vw[q]));
            o0 = __ffma2_rn(make_float2(pw[q].x, pw[q].x), vv, o0);
            o1 = __ffma2_rn(make_float2(pw[q].y, pw[q].y), vv, o1);
          }
        }
        for (; r < n; r++) {
          const uint32_t vw = *reinterpret_cast<const uint32_t*>(vb + (size_t)r * (2 * D));
          const float2 pw = *reinterpret_cast<const float2*>(pp + (size_t)r * G);
          const float2 vv = make_float2(bf_lo(vw), bf_hi(vw));
          o0 = __ffma2_rn(make_float2(pw.x, pw.x), vv, o0);
          o1 = __ffma2_rn(make_float2(pw.y, pw.y), vv, o1);
        }
        const int ha = 2 * hp, hb = 2 * hp + 1;
        const float la = stat[ha * 2], lb = stat[hb * 2];
        *reinterpret_cast<float2*>(a.part_o + ((size_t)s * a.nq + hq0 + ha) * D + 2 * dp) =
            make_float2(__fdiv_rn(o0.x, la), __fdiv_rn(o0.y, la));
        *reinterpret_cast<float2*>(a.part_o + ((size_t)s * a.nq + hq0 + hb) * D + 2 * dp) =
            make_float2(__fdiv_rn(o1.x, lb), __fdiv_rn(o1.y, lb));
        if (dp == 0) {
          a.part_lse[(size_t)s * a.nq + hq0 + ha] = __fadd_rn(spark_log(la), stat[ha * 2 + 1]);
          a.part_lse[(size_t)s * a.nq + hq0 + hb] = __fadd_rn(spark_log(lb), stat[hb * 2 + 1]);
        }
      }
    } else {
      // a copy never landed: report it, give the copies a last bounded wait before the
      // shared memory is released, publish an empty split
      if (tid == 0) {
        if (a.error) atomicExch(a.error, 2);
        mbar_wait(kbar, 0);
        mbar_wait(vbar, 0);
      }
      ok = false;
    }
  }
  if (!ok) {
    if (n > 0 && T > a.t_alloc && tid == 0 && a.error) atomicExch(a.error, 1);
    for (int i = tid; i < G * D; i += kWideThreads) a.part_o[((size_t)s * a.nq + hq0) * D + i] = 0.0f;
    if (tid < G) a.part_lse[(size_t)s * a.nq + hq0 + tid] = ninf;
  }

  if (a.out == nullptr) return;
  // ---- fused combine: the last split CTA of this kv head merges its four q heads
  __threadfence();
  __syncthreads();
  if (tid == 0) flag[0] = (atomicAdd(&a.counters[hk], 1) == a.splits - 1);
  __syncthreads();
  if (!flag[0]) return;
  __threadfence();
  attn_merge_heads<D, G, kWideThreads>(a.part_o, a.part_lse, a.splits, a.nq, hq0, a.out, wn, stat, kbuf,
                                       (size_t)TA * (4 * D));
  if (tid == 0) a.counters[hk] = 0;
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

// Standalone combine for groups of 4 query heads (splits <= 256): same helper as the
// fused path.  grid = nq / 4, 128 threads.
__global__ void __launch_bounds__(128) attn_combine4_kernel(const CombineArgs a) {
  extern __shared__ __align__(16) unsigned char smem_c[];
  float* wn = reinterpret_cast<float*>(smem_c);   // [4][kAttnMaxFusedSplits]
  float* mx = wn + 4 * kAttnMaxFusedSplits;      // [4][2] (+ pad)
  unsigned char* buf = reinterpret_cast<unsigned char*>(mx + 8);
  pdl_launch_dependents();
  pdl_wait();
  attn_merge_heads<128, 4>(a.part_o, a.part_lse, a.splits, a.nq, blockIdx.x * 4, a.out, wn, mx, buf, 64 * 1024);
}

}  // namespace spark
