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
// Arithmetic (canonical order, mirrored by the CPU oracle):
//   * once per call the activation x is staged in shared memory as exact 16-bit
//     fixed point per 32-element block: M = max |x_j|, S = 14 - floor(log2 M),
//     X_j = rint(x_j * 2^S), sx = 2^-S, C = 8 * sum X_j (blocks with M < 2^-100
//     are zero).  X_j is split into a signed high byte and an unsigned low byte,
//     packed four elements per 32-bit word in the order the nibble words need;
//   * per weight block: P = sum_j (q_j - 8) X_j is computed exactly with dp4a
//     (low nibbles v & 0x0f0f0f0f, high nibbles v & 0xf0f0f0f0 = 16 q), then
//     lane acc = fma(fp32(d) * sx, float(P), acc) -- |P| < 2^24, so float(P) is exact;
//   * the 16 per-lane row sums are combined with an xor butterfly (8, 4, 2, 1) and
//     rounded to bf16.
#pragma once

#include "common.cuh"

namespace spark {

// ------------------------------------------------------------------ fixed-point x staging
// Shared-memory layout of one staged activation row with nb blocks:
//   xq  uint4 [4][nb]: xq[w*nb + b] = (hi bytes of X[4w..4w+3], lo bytes of X[4w..4w+3],
//                                     hi bytes of X[16+4w..16+4w+3], lo bytes of the same)
//   xm  float2 [nb]:   (sx, C as int bits)
constexpr float kStageMinMax = 7.888609052210118e-31f;  // 2^-100

// Stage block b (the canonical fixed point above) with its 32 elements spread over the 4
// consecutive lanes of a quad (lane c: elements 8c .. 8c+7): every lane of the warp calls
// it, a lane without a block with valid = false and zeros.  The maximum and the integer
// sum are exact in any order, so the staged words do not depend on the split.
__device__ __forceinline__ void stage_block_q4(const float (&v)[8], bool valid, uint4* xq, float2* xm, int nb, int b,
                                               int c) {
  float M = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; j++) M = fmaxf(M, fabsf(v[j]));
  M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 1));
  M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 2));
  int X[8];
  float sx = 1.0f;
  int sum = 0;
  if (M >= kStageMinMax && M != __int_as_float(0x7f800000)) {
    const int e = (int)((__float_as_uint(M) >> 23) & 0xffu) - 127;
    const int S = 14 - e;
    const float sc = __uint_as_float((uint32_t)(S + 127) << 23);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      X[j] = __float2int_rn(__fmul_rn(v[j], sc));
      sum += X[j];
    }
    sx = __uint_as_float((uint32_t)(127 - S) << 23);
  } else {
#pragma unroll
    for (int j = 0; j < 8; j++) X[j] = 0;
  }
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);
  sum += __shfl_xor_sync(0xffffffffu, sum, 2);
  if (valid) {
    // elements 4q .. 4q+3, q = 2c, 2c+1: word q (hi, lo halves) for q < 4, else the
    // (hi, lo) halves of word q - 4 for elements 16 + 4 (q - 4) ..
#pragma unroll
    for (int t2 = 0; t2 < 2; t2++) {
      const int q = 2 * c + t2;
      uint32_t hi = 0, lo = 0;
#pragma unroll
      for (int t = 0; t < 4; t++) {
        const int a = X[4 * t2 + t];
        hi |= (uint32_t)((a >> 8) & 0xff) << (8 * t);
        lo |= (uint32_t)(a & 0xff) << (8 * t);
      }
      reinterpret_cast<uint2*>(xq + (q & 3) * nb + b)[q >> 2] = make_uint2(hi, lo);
    }
    if (c == 0) xm[b] = make_float2(sx, __int_as_float(8 * sum));
  }
}

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// exact integer dot product of one Q4_0 block with its staged x block (before -C):
// xb points at xq[b]; consecutive words of the block are `stride` uint4 apart
__device__ __forceinline__ int block_int_dot(const uint4 q, const uint4* __restrict__ xb, int stride) {
  const uint32_t words[4] = {q.x, q.y, q.z, q.w};
  int A = 0, Cc = 0;
  uint32_t B = 0, D = 0;
#pragma unroll
  for (int w = 0; w < 4; w++) {
    const uint32_t lo = words[w] & 0x0f0f0f0fu, hi = words[w] & 0xf0f0f0f0u;
    const uint4 xw = xb[w * stride];
    A = dp4a_us(lo, xw.x, A);
    B = __dp4a(lo, xw.y, B);
    Cc = dp4a_us(hi, xw.z, Cc);
    D = __dp4a(hi, xw.w, D);
  }
  return A * 256 + (int)B + Cc * 16 + (int)(D >> 4);
}

// lane accumulation of one block: acc = fma(fp32(d) * sx, float(P - C), acc)
__device__ __forceinline__ float block_accum(float acc, uint16_t d, const uint4 q, const uint4* __restrict__ xb,
                                             int stride, const float2 m) {
  const int P = block_int_dot(q, xb, stride) - __float_as_int(m.y);
  return __fmaf_rn(__fmul_rn(h2f(d), m.x), __int2float_rn(P), acc);
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
  int* error;  // device error word (ring kernel: bounded-wait timeouts), may be null
};

// ------------------------------------------------------------------ prologues
// Prologues.  sync(n) is the barrier among the n staging threads: all threads of
// the CTA for the register-direct kernel (n == blockDim.x), the consumer warps
// (named barrier 1) for the ring kernel.
__device__ __forceinline__ void staging_sync(int n) {
  if (n == (int)blockDim.x)
    __syncthreads();
  else
    asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory");
}
struct ProPlain {
  static constexpr bool kNorm = false;
  __device__ static void sync(int n) { staging_sync(n); }
};
struct ProNorm {
  static constexpr bool kNorm = true;
  __device__ static void sync(int n) { staging_sync(n); }
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
  __device__ static void store_row(const GemvArgs& g, EpiState& st, int bt, int r, float s) {
    g.y[(size_t)bt * g.n + r] = f2bf(s);
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
  __device__ static void store_row(const GemvArgs& g, EpiState& st, int bt, int r, float s) {
    uint16_t b = f2bf(s);
    g.y[(size_t)bt * g.n + r] = b;
    unsigned long long k = key(b, r);
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
  // q/k pairs rotate (i, i + D/2) of one head (neox).  v pairs are
  // (vbase + t, vbase + t + nkv*D/2): any pairing works for v, and this one keeps
  // each side of a run of pairs contiguous in memory.
  __device__ static int num_pairs(const GemvArgs& g) { return g.n >> 1; }
  __device__ static void rows(const GemvArgs& g, int p, int& r0, int& r1) {
    const int half = g.head_dim >> 1;
    const int rot_pairs = (g.nq + g.nkv) * half;
    if (p < rot_pairs) {
      int h = p / half, i = p - h * half;
      r0 = h * g.head_dim + i;
      r1 = r0 + half;
    } else {
      r0 = (g.nq + g.nkv) * g.head_dim + (p - rot_pairs);
      r1 = r0 + g.nkv * half;
    }
  }
  __device__ static int64_t position(const GemvArgs& g) { return g.pos64 ? g.pos64[0] : (int64_t)g.pos32[0]; }
  __device__ static int64_t slot(const GemvArgs& g, int64_t pos) {
    if (g.slot_mapping) return g.slot_mapping[0];
    int64_t blk = pos / g.block_size;
    return (int64_t)g.block_table[blk] * g.block_size + (pos - blk * g.block_size);
  }
  __device__ static void store_v(const GemvArgs& g, int64_t sl, int r, float s) {
    const int D = g.head_dim;
    int e = r - (g.nq + g.nkv) * D;
    int hk = e / D, dd = e - hk * D;
    int64_t blk = sl / g.block_size, off = sl - blk * g.block_size;
    g.v_cache[((blk * g.nkv + hk) * g.block_size + off) * D + dd] = f2bf(s);
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
        store_v(g, sl, r0, s0);
        store_v(g, sl, r1, s1);
      }
    }
  }
  template <int BATCH>
  __device__ static void finish(const GemvArgs& g, EpiState& st, unsigned long long* red) {}
};

// ------------------------------------------------------------------ x staging
// smem per batch row: xq (64 * nb bytes) then xm (8 * nb bytes); after all batch
// rows: red (40 floats) and, for the norm prologue, slin (k floats).
// Plain: x bf16 [batch][k].  Norm: s = a + b, res_out = bf16(s) (CTA 0), ss by
// warp 0 in the canonical 32-lane order, x = bf16((s * inv) * gamma).
template <class Pro, int BATCH>
__device__ __forceinline__ void stage_x(const GemvArgs& g, unsigned char* smem, float* red, float* slin, int tid,
                                        int nthreads) {
  const int k = g.k, nb = k >> 5;
  if constexpr (!Pro::kNorm) {
    for (int bt = 0; bt < BATCH; bt++) {
      uint4* xq = reinterpret_cast<uint4*>(smem + (size_t)bt * 72 * nb);
      float2* xm = reinterpret_cast<float2*>(smem + (size_t)bt * 72 * nb + 64 * nb);
      const uint4* src = reinterpret_cast<const uint4*>(g.x + (size_t)bt * k);
      // item = 4 b + c: lane c of block b's quad (nthreads is a multiple of 32, so every
      // lane of a warp takes the same number of rounds); the loads of 4 rounds first
      for (int base = 0; base < 4 * nb; base += 4 * nthreads) {
        uint4 u[4];
#pragma unroll
        for (int rr = 0; rr < 4; rr++) {
          const int item = base + rr * nthreads + tid;
          u[rr] = (item < 4 * nb && bt < g.batch) ? src[item] : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int rr = 0; rr < 4; rr++) {
          const int item = base + rr * nthreads + tid;
          if (base + rr * nthreads >= 4 * nb) break;  // (warp-uniform)
          float v[8];
          const uint32_t w4[4] = {u[rr].x, u[rr].y, u[rr].z, u[rr].w};
#pragma unroll
          for (int t = 0; t < 4; t++) {
            v[2 * t] = bf_lo(w4[t]);
            v[2 * t + 1] = bf_hi(w4[t]);
          }
          stage_block_q4(v, item < 4 * nb, xq, xm, nb, item >> 2, item & 3);
        }
      }
    }
  } else {
    const uint16_t* arow = g.embed ? g.embed + (size_t)g.token[0] * k : g.a;
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(arow);
    const uint32_t* pb = reinterpret_cast<const uint32_t*>(g.b);
    const bool write_res = (g.res_out != nullptr) && blockIdx.x == 0;
    for (int i = tid; i < (k >> 1); i += nthreads) {
      const uint32_t va = pa[i];
      float s0, s1;
      if (pb) {
        const uint32_t vb = pb[i];
        s0 = __fadd_rn(bf_lo(va), bf_lo(vb));
        s1 = __fadd_rn(bf_hi(va), bf_hi(vb));
      } else {
        s0 = bf_lo(va);
        s1 = bf_hi(va);
      }
      reinterpret_cast<float2*>(slin)[i] = make_float2(s0, s1);
      if (write_res) reinterpret_cast<uint32_t*>(g.res_out)[i] = (uint32_t)f2bf(s0) | ((uint32_t)f2bf(s1) << 16);
    }
    Pro::sync(nthreads);
    if (tid < 32) {
      float acc = 0.0f;
#pragma unroll 8
      for (int i = tid; i < k; i += 32) {
        const float sv = slin[i];
        acc = __fadd_rn(acc, __fmul_rn(sv, sv));
      }
      acc = butterfly_sum<32>(acc);
      if (tid == 0) red[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(acc, g.inv_k), g.eps)));
    }
    Pro::sync(nthreads);
    const float inv = red[0];
    uint4* xq = reinterpret_cast<uint4*>(smem);
    float2* xm = reinterpret_cast<float2*>(smem + 64 * nb);
    const uint32_t* pg = reinterpret_cast<const uint32_t*>(g.gamma);
    for (int base = 0; base < 4 * nb; base += 4 * nthreads) {  // 4 lanes per block, as above
      uint32_t gw[4][4];  // gamma pairs of 4 rounds, loaded first
#pragma unroll
      for (int rr = 0; rr < 4; rr++) {
        const int item = base + rr * nthreads + tid;
#pragma unroll
        for (int j = 0; j < 4; j++) gw[rr][j] = item < 4 * nb ? pg[4 * item + j] : 0u;
      }
#pragma unroll
      for (int rr = 0; rr < 4; rr++) {
        const int item = base + rr * nthreads + tid;
        if (base + rr * nthreads >= 4 * nb) break;  // (warp-uniform)
        const bool valid = item < 4 * nb;
        float v[8];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          v[2 * j] = 0.0f;
          v[2 * j + 1] = 0.0f;
          if (valid) {
            const float2 sv = reinterpret_cast<const float2*>(slin)[4 * item + j];
            v[2 * j] = bf2f(f2bf(__fmul_rn(__fmul_rn(sv.x, inv), bf_lo(gw[rr][j]))));
            v[2 * j + 1] = bf2f(f2bf(__fmul_rn(__fmul_rn(sv.y, inv), bf_hi(gw[rr][j]))));
          }
        }
        stage_block_q4(v, valid, xq, xm, nb, item >> 2, item & 3);
      }
    }
  }
  Pro::sync(nthreads);
}

// ------------------------------------------------------------------ the kernel
// NBL: blocks per lane loaded per chunk (compile time); a lane walks its blocks
// l, l+16, ... in ascending order, NBL at a time.  Each half warp owns a row
// pair; a warp works on two adjacent pairs ("duo").  Duos are dealt to warps
// interleaved across CTAs so that every SM gets an even share.
template <class Pro, class Epi, int BATCH, int NBL>
__global__ void __launch_bounds__(256) q4_gemv_kernel(const GemvArgs g) {
  extern __shared__ __align__(16) unsigned char smem_u8[];
  const int nb = g.k >> 5;
  float* red = reinterpret_cast<float*>(smem_u8 + (size_t)BATCH * 72 * nb);
  float* slin = red + 40;

  pdl_launch_dependents();
  pdl_wait();
  stage_x<Pro, BATCH>(g, smem_u8, red, slin, threadIdx.x, blockDim.x);

  const int lane = threadIdx.x & 31, hl = lane & 15, half = lane >> 4, warp = threadIdx.x >> 5;
  const int npairs = Epi::num_pairs(g);
  const int warps_total = gridDim.x * (blockDim.x >> 5);
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
#pragma unroll
          for (int bt = 0; bt < BATCH; bt++) {
            const uint4* xq = reinterpret_cast<const uint4*>(smem_u8 + (size_t)bt * 72 * nb);
            const float2 m = reinterpret_cast<const float2*>(smem_u8 + (size_t)bt * 72 * nb + 64 * nb)[b];
            acc0[bt] = block_accum(acc0[bt], s0[j], wq0[j], xq + b, nb, m);
            acc1[bt] = block_accum(acc1[bt], s1[j], wq1[j], xq + b, nb, m);
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
  Epi::template finish<BATCH>(g, st, reinterpret_cast<unsigned long long*>(red + 8));
}

}  // namespace spark
