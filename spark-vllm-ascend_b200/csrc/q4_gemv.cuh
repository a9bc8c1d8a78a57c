// q4_gemv.cuh -- Q4_0 block-dequant GEMV for batch-1 (and batch <= 8) decode on sm_100a.
//
// Reference: kernels/linear.py:17-200 (GemvStage.calculate) and its callers
// NativeLinear.execute_o/execute_down (linear.py:339-370), NativeUp.execute
// (linear.py:585-611) and FusedQkvStage.execute_fused (qkv.py:201-236).
//
// Weight layout in HBM (lossless split of gguf Q4_0 blocks):
//   qs : uint8  [N][K/2]   the 16 nibble bytes of each 32-weight block, gguf order
//                          (byte j: low nibble = element j, high nibble = element j+16)
//   d  : fp16   [N][K/32]  the block scale
// A row is read by 16 lanes (a half warp) with 128-bit loads: lane l owns blocks
// l, l+16, ... so one load instruction of a half warp covers 256 contiguous bytes.
//
// Arithmetic per block (canonical order, mirrored by the CPU oracle):
//   nibble -> exact (q - 8) in fp32 with one LOP3 per value (a magic exponent chosen
//   per nibble position) and one packed f32x2 subtract per pair, then packed f32x2
//   FMAs: lane .x accumulates elements 0..15, lane .y elements 16..31, in ascending
//   order; block sum = .x + .y; row acc = fma(d, block sum, acc).  The 16 per-lane
//   row sums are combined with an xor butterfly (8, 4, 2, 1) and rounded to bf16.
#pragma once

#include "common.cuh"

namespace spark {

// x staging in shared memory (fp32), per batch row: float4 slot (w*2+h)*nb + b holds
// (x[32b+4w+2h], x[32b+4w+2h+16], x[32b+4w+2h+1], x[32b+4w+2h+17]), i.e. the two
// (element, element+16) pairs that word w of block b multiplies with.
__device__ __forceinline__ int xs_index(int e, int nb) {
  int b = e >> 5, j = e & 31, hi = j >> 4, lo = j & 15;
  int w = lo >> 2, k = lo & 3, h = k >> 1;
  return (((w * 2 + h) * nb + b) << 2) + ((k & 1) << 1) + hi;
}

// dequantize one 32-bit word (8 nibbles) into 4 exact (q-8) pairs
__device__ __forceinline__ void dequant_word(uint32_t v, float2& w0, float2& w1, float2& w2, float2& w3) {
  const uint32_t u = v >> 12;
  w0 = make_float2(__uint_as_float((v & 0x0000000fu) | 0x4b000000u), __uint_as_float((v & 0x000000f0u) | 0x49000000u));
  w1 = make_float2(__uint_as_float((v & 0x00000f00u) | 0x47000000u), __uint_as_float((v & 0x0000f000u) | 0x45000000u));
  w2 = make_float2(__uint_as_float((v & 0x000f0000u) | 0x43000000u), __uint_as_float((u & 0x00000f00u) | 0x47000000u));
  w3 = make_float2(__uint_as_float((u & 0x0000f000u) | 0x45000000u), __uint_as_float((u & 0x000f0000u) | 0x43000000u));
  w0 = __fadd2_rn(w0, make_float2(-8388616.0f, -524296.0f));
  w1 = __fadd2_rn(w1, make_float2(-32776.0f, -2056.0f));
  w2 = __fadd2_rn(w2, make_float2(-136.0f, -32776.0f));
  w3 = __fadd2_rn(w3, make_float2(-2056.0f, -136.0f));
}

// block sum (a0 + a1) of one 32-weight block against staged x
__device__ __forceinline__ float block_dot(const uint4 q, const float4* __restrict__ xs, int nb, int b) {
  float2 a = make_float2(0.0f, 0.0f);
  const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int w = 0; w < 4; w++) {
    float2 w0, w1, w2, w3;
    dequant_word(words[w], w0, w1, w2, w3);
    const float4 x01 = xs[(w * 2 + 0) * nb + b];
    const float4 x23 = xs[(w * 2 + 1) * nb + b];
    a = __ffma2_rn(w0, make_float2(x01.x, x01.y), a);
    a = __ffma2_rn(w1, make_float2(x01.z, x01.w), a);
    a = __ffma2_rn(w2, make_float2(x23.x, x23.y), a);
    a = __ffma2_rn(w3, make_float2(x23.z, x23.w), a);
  }
  return __fadd_rn(a.x, a.y);
}

// ------------------------------------------------------------------ argument block
struct GemvArgs {
  // weights
  const uint8_t* qs;
  const uint16_t* d;
  int n, k;
  int batch;
  // prologue: plain x, or fused add + RMSNorm of (a + b)
  const uint16_t* x;      // bf16 [batch][k]           (plain)
  const uint16_t* a;      // bf16 [k]                   (norm)
  const uint16_t* b;      // bf16 [k] or null           (norm)
  const uint16_t* gamma;  // bf16 [k]                   (norm)
  uint16_t* res_out;      // bf16 [k] or null           (norm: bf16(a+b), written by CTA 0)
  const uint16_t* embed;  // bf16 [vocab][k] or null    (norm: a = embed[token[0]])
  const int32_t* token;
  float eps, inv_k;
  // outputs
  uint16_t* y;  // bf16 [batch][n] (plain / argmax logits) or q/mid output
  // rope + kv store epilogue
  int nq, nkv, head_dim, block_size;
  const uint16_t* cos_sin;   // bf16 [max_pos][head_dim]
  const int64_t* pos64;      // position (one of pos64 / pos32)
  const int32_t* pos32;
  const int32_t* block_table;
  const int64_t* slot_mapping;  // optional; overrides block_table
  uint16_t* k_cache;  // bf16 [blocks][nkv][block_size][head_dim]
  uint16_t* v_cache;
  // silu-mul epilogue: gate rows [0, n/2), up rows [n/2, n)
  // argmax epilogue
  unsigned long long* argmax_key;
};

// ------------------------------------------------------------------ prologues
struct ProPlain {
  static constexpr bool kNorm = false;
};
struct ProNorm {
  static constexpr bool kNorm = true;
};

// ------------------------------------------------------------------ epilogues
struct EpiState {
  unsigned long long best[8];  // argmax epilogue: running key per batch row
};

struct EpiPlain {
  __device__ static int num_pairs(const GemvArgs& g) { return g.n >> 1; }
  __device__ static void rows(const GemvArgs& g, int p, int& r0, int& r1) {
    r0 = 2 * p;
    r1 = 2 * p + 1;
  }
  __device__ static void store(const GemvArgs& g, EpiState& st, int bt, int p, int r0, int r1, float s0, float s1) {
    uint32_t packed = (uint32_t)f2bf(s0) | ((uint32_t)f2bf(s1) << 16);
    *reinterpret_cast<uint32_t*>(g.y + (size_t)bt * g.n + r0) = packed;
  }
  template <int BATCH>
  __device__ static void finish(const GemvArgs& g, EpiState& st, unsigned long long* red) {}
};

// Logits + greedy argmax: largest bf16 logit, lowest index on ties.  Keys are
// (order-preserving bits << 32) | (~index); each CTA reduces its rows and issues
// one atomicMax per batch row, so the result does not depend on CTA order.
struct EpiArgmax {
  __device__ static int num_pairs(const GemvArgs& g) { return g.n >> 1; }
  __device__ static void rows(const GemvArgs& g, int p, int& r0, int& r1) {
    r0 = 2 * p;
    r1 = 2 * p + 1;
  }
  __device__ static unsigned long long key(uint16_t bits, int idx) {
    uint32_t u = (uint32_t)bits << 16;
    uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
  }
  __device__ static void store(const GemvArgs& g, EpiState& st, int bt, int p, int r0, int r1, float s0, float s1) {
    uint16_t b0 = f2bf(s0), b1 = f2bf(s1);
    *reinterpret_cast<uint32_t*>(g.y + (size_t)bt * g.n + r0) = (uint32_t)b0 | ((uint32_t)b1 << 16);
    unsigned long long k0 = key(b0, r0), k1 = key(b1, r1);
    unsigned long long k = k0 > k1 ? k0 : k1;
    if (k > st.best[bt]) st.best[bt] = k;
  }
  template <int BATCH>
  __device__ static void finish(const GemvArgs& g, EpiState& st, unsigned long long* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int bt = 0; bt < BATCH; bt++) {
      unsigned long long k = st.best[bt];
#pragma unroll
      for (int off = 16; off >= 1; off /= 2) {
        unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
        k = o > k ? o : k;
      }
      if (lane == 0) red[warp] = k;
      __syncthreads();
      if (threadIdx.x == 0) {
        unsigned long long m = 0;
        for (int w = 0; w < nw; w++) m = red[w] > m ? red[w] : m;
        if (m) atomicMax(g.argmax_key + bt, m);
      }
      __syncthreads();
    }
  }
};

struct EpiSiluMul {
  // pair p -> (gate row p, up row n/2 + p); output mid[p]
  __device__ static int num_pairs(const GemvArgs& g) { return g.n >> 1; }
  __device__ static void rows(const GemvArgs& g, int p, int& r0, int& r1) {
    r0 = p;
    r1 = (g.n >> 1) + p;
  }
  __device__ static void store(const GemvArgs& g, EpiState& st, int bt, int p, int r0, int r1, float s0, float s1) {
    float gf = bf2f(f2bf(s0));
    float uf = bf2f(f2bf(s1));
    float act = bf2f(f2bf(__fdiv_rn(gf, __fadd_rn(1.0f, spark_exp(-gf)))));
    g.y[(size_t)bt * (g.n >> 1) + p] = f2bf(__fmul_rn(act, uf));
  }
  template <int BATCH>
  __device__ static void finish(const GemvArgs& g, EpiState& st, unsigned long long* red) {}
};

struct EpiRope {
  // rows: q heads [0, nq*D), k heads [nq*D, (nq+nkv)*D), v heads after.
  // q/k pairs rotate (i, i + D/2) of one head (neox); v pairs are adjacent rows.
  __device__ static int num_pairs(const GemvArgs& g) { return g.n >> 1; }
  __device__ static void rows(const GemvArgs& g, int p, int& r0, int& r1) {
    const int half = g.head_dim >> 1;
    const int rot_pairs = (g.nq + g.nkv) * half;
    if (p < rot_pairs) {
      int h = p / half, i = p - h * half;
      r0 = h * g.head_dim + i;
      r1 = r0 + half;
    } else {
      r0 = (g.nq + g.nkv) * g.head_dim + 2 * (p - rot_pairs);
      r1 = r0 + 1;
    }
  }
  __device__ static int64_t position(const GemvArgs& g) { return g.pos64 ? g.pos64[0] : (int64_t)g.pos32[0]; }
  __device__ static int64_t slot(const GemvArgs& g, int64_t pos) {
    if (g.slot_mapping) return g.slot_mapping[0];
    int64_t blk = pos / g.block_size;
    return (int64_t)g.block_table[blk] * g.block_size + (pos - blk * g.block_size);
  }
  __device__ static void store(const GemvArgs& g, EpiState& st, int bt, int p, int r0, int r1, float s0, float s1) {
    const int D = g.head_dim, half = D >> 1;
    const int rot_pairs = (g.nq + g.nkv) * half;
    const int64_t pos = position(g);
    if (p < rot_pairs) {
      int h = p / half, i = p - h * half;
      float a = bf2f(f2bf(s0)), b = bf2f(f2bf(s1));
      const uint16_t* cs = g.cos_sin + (size_t)pos * D;
      float c = bf2f(cs[i]), s = bf2f(cs[i + half]);
      float u = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
      float v = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
      uint16_t ub = f2bf(u), vb = f2bf(v);
      if (h < g.nq) {
        g.y[(size_t)h * D + i] = ub;
        g.y[(size_t)h * D + i + half] = vb;
      } else {
        int64_t sl = slot(g, pos);
        if (sl >= 0) {
          int hk = h - g.nq;
          int64_t blk = sl / g.block_size, off = sl - blk * g.block_size;
          uint16_t* dst = g.k_cache + ((blk * g.nkv + hk) * g.block_size + off) * D;
          dst[i] = ub;
          dst[i + half] = vb;
        }
      }
    } else {
      int64_t sl = slot(g, pos);
      if (sl >= 0) {
        int e = r0 - (g.nq + g.nkv) * D;
        int hk = e / D, dd = e - hk * D;
        int64_t blk = sl / g.block_size, off = sl - blk * g.block_size;
        uint16_t* dst = g.v_cache + ((blk * g.nkv + hk) * g.block_size + off) * D + dd;
        *reinterpret_cast<uint32_t*>(dst) = (uint32_t)f2bf(s0) | ((uint32_t)f2bf(s1) << 16);
      }
    }
  }
  template <int BATCH>
  __device__ static void finish(const GemvArgs& g, EpiState& st, unsigned long long* red) {}
};

// ------------------------------------------------------------------ x staging
// Plain: x bf16 [batch][k] -> xs.  Norm: s = a + b, res_out = bf16(s) (CTA 0),
// ss by warp 0 in the canonical 32-lane order, y = bf16((s * inv) * gamma).
template <class Pro, int BATCH>
__device__ __forceinline__ void stage_x(const GemvArgs& g, float* xs, float* red) {
  const int k = g.k, nb = k >> 5;
  if constexpr (!Pro::kNorm) {
    for (int bt = 0; bt < BATCH; bt++) {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(g.x + (size_t)bt * k);
      float* dst = xs + (size_t)bt * k;
      for (int i = threadIdx.x; i < (k >> 1); i += blockDim.x) {
        uint32_t v = bt < g.batch ? src[i] : 0u;
        dst[xs_index(2 * i, nb)] = bf_lo(v);
        dst[xs_index(2 * i + 1, nb)] = bf_hi(v);
      }
    }
    __syncthreads();
  } else {
    // phase 1: s = a + b into xs (fp32), residual out
    const uint16_t* arow = g.embed ? g.embed + (size_t)g.token[0] * k : g.a;
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(arow);
    const uint32_t* pb = reinterpret_cast<const uint32_t*>(g.b);
    const bool write_res = (g.res_out != nullptr) && blockIdx.x == 0;
    for (int i = threadIdx.x; i < (k >> 1); i += blockDim.x) {
      uint32_t va = pa[i];
      float s0, s1;
      if (pb) {
        uint32_t vb = pb[i];
        s0 = __fadd_rn(bf_lo(va), bf_lo(vb));
        s1 = __fadd_rn(bf_hi(va), bf_hi(vb));
      } else {
        s0 = bf_lo(va);
        s1 = bf_hi(va);
      }
      xs[xs_index(2 * i, nb)] = s0;
      xs[xs_index(2 * i + 1, nb)] = s1;
      if (write_res)
        reinterpret_cast<uint32_t*>(g.res_out)[i] = (uint32_t)f2bf(s0) | ((uint32_t)f2bf(s1) << 16);
    }
    __syncthreads();
    // phase 2: canonical sum of squares (warp 0)
    if (threadIdx.x < 32) {
      float acc = 0.0f;
      for (int i = threadIdx.x; i < k; i += 32) {
        float s = xs[xs_index(i, nb)];
        acc = __fadd_rn(acc, __fmul_rn(s, s));
      }
      acc = butterfly_sum<32>(acc);
      if (threadIdx.x == 0) {
        float root = __fsqrt_rn(__fadd_rn(__fmul_rn(acc, g.inv_k), g.eps));
        red[0] = __fdiv_rn(1.0f, root);
      }
    }
    __syncthreads();
    // phase 3: y = bf16((s * inv) * gamma) in place
    const float inv = red[0];
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      int idx = xs_index(i, nb);
      xs[idx] = bf2f(f2bf(__fmul_rn(__fmul_rn(xs[idx], inv), bf2f(g.gamma[i]))));
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ the kernel
// NBL: blocks per lane loaded per chunk (compile time); a lane walks its blocks
// l, l+16, ... in ascending order, NBL at a time.  Each half warp owns a row
// pair; a warp works on two adjacent pairs ("duo").  Duos are dealt to warps
// interleaved across CTAs so that every SM gets an even share.
template <class Pro, class Epi, int BATCH, int NBL>
__global__ void __launch_bounds__(256) q4_gemv_kernel(const GemvArgs g) {
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;
  float* red = smem + (size_t)BATCH * g.k;

  pdl_launch_dependents();
  pdl_wait();
  stage_x<Pro, BATCH>(g, xs, red);

  const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4, warp = threadIdx.x >> 5;
  const int nb = g.k >> 5;
  const int npairs = Epi::num_pairs(g);
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  const float4* xs4 = reinterpret_cast<const float4*>(xs);
  const size_t row_bytes = (size_t)g.k >> 1;
  const int my_blocks = nb > hl ? (nb - hl + 15) >> 4 : 0;
  EpiState st;
#pragma unroll
  for (int bt = 0; bt < 8; bt++) st.best[bt] = 0ull;

  for (int duo = warp * gridDim.x + blockIdx.x; duo * 2 < npairs; duo += warps_total) {
    const int p = duo * 2 + half;
    const bool active = p < npairs;
    int r0 = 0, r1 = 0;
    if (active) Epi::rows(g, p, r0, r1);
    const uint8_t* q0 = g.qs + (size_t)r0 * row_bytes;
    const uint8_t* q1 = g.qs + (size_t)r1 * row_bytes;
    const uint16_t* d0 = g.d + (size_t)r0 * nb;
    const uint16_t* d1 = g.d + (size_t)r1 * nb;
    const int nblk = active ? my_blocks : 0;

    float acc0[BATCH], acc1[BATCH];
#pragma unroll
    for (int bt = 0; bt < BATCH; bt++) acc0[bt] = acc1[bt] = 0.0f;

    for (int j0 = 0; j0 < nblk; j0 += NBL) {
      uint4 wq0[NBL], wq1[NBL];
      uint16_t s0[NBL], s1[NBL];
#pragma unroll
      for (int j = 0; j < NBL; j++) {
        const int b = hl + 16 * (j0 + j);
        if (j0 + j < nblk) {
          wq0[j] = ldg_stream(q0 + (size_t)b * 16);
          wq1[j] = ldg_stream(q1 + (size_t)b * 16);
          s0[j] = ldg_u16_stream(d0 + b);
          s1[j] = ldg_u16_stream(d1 + b);
        }
      }
#pragma unroll
      for (int j = 0; j < NBL; j++) {
        const int b = hl + 16 * (j0 + j);
        if (j0 + j < nblk) {
          const float sc0 = h2f(s0[j]), sc1 = h2f(s1[j]);
#pragma unroll
          for (int bt = 0; bt < BATCH; bt++) {
            const float4* xb = xs4 + (size_t)bt * (g.k >> 2);
            acc0[bt] = __fmaf_rn(sc0, block_dot(wq0[j], xb, nb, b), acc0[bt]);
            acc1[bt] = __fmaf_rn(sc1, block_dot(wq1[j], xb, nb, b), acc1[bt]);
          }
        }
      }
    }
#pragma unroll
    for (int bt = 0; bt < BATCH; bt++) {
      acc0[bt] = butterfly_sum<16>(acc0[bt]);
      acc1[bt] = butterfly_sum<16>(acc1[bt]);
    }
    if (active && hl == 0) {
#pragma unroll
      for (int bt = 0; bt < BATCH; bt++)
        if (bt < g.batch) Epi::store(g, st, bt, p, r0, r1, acc0[bt], acc1[bt]);
    }
  }
  Epi::template finish<BATCH>(g, st, reinterpret_cast<unsigned long long*>(red + 4));
}

}  // namespace spark
