// step_kernel.cuh -- the persistent decode-step kernel (one cooperative launch per
// decode step, one CTA per SM).
//
// A launch runs a program of stages (SparkStage, include/spark_b200.h): GEMV stages
// over Q4_0 weights in the T16 layout, and split-KV attention stages.  Every CTA has
// a producer warp and 12 consumer warps:
//
//  * the producer (one thread) walks the whole program ahead of the consumers and
//    streams, with cp.async.bulk, every byte its CTA will read from HBM into a
//    byte ring in shared memory: the T16 units of its share of each GEMV stage and
//    the K / V page runs of its attention split.  It never waits on other CTAs, so
//    weight traffic keeps flowing while the consumers sit at a stage barrier.
//  * the consumers execute the stages in order.  A stage whose input comes from the
//    previous stage waits (bounded) until every CTA has arrived on that stage's
//    global counter, stages its input vector, works through its ring units, runs the
//    stage epilogue and arrives on its own counter.
//
// GEMV arithmetic: a Q4_0 block's integer dot product sum_j (q_j - 8) X_j runs on
// the tensor cores as mma.m16n8k32 (u8 nibbles of 16 rows x s8 activation digits,
// X = 256 h + l in B columns 0 and 1, -8 sum X through the accumulator input), then
// acc = fma(d * sx, P, acc) per row and block exactly as the oracle's T16 order.
//
// All waits are bounded (globaltimer, 2 s): a wait that runs out records
// SPARK_ERR_LAUNCH in the error word, raises the abort flag and the kernel drains
// its copies and returns.  Counters are left non-zero after an abort; the host
// resets them (spark_step_run's caller zeroes io->counters).
#pragma once

#include "common.cuh"
#include "q4_gemv_ring.cuh"
#include "spark_b200.h"

namespace spark {
namespace step {

constexpr int kWarps = 12;                 // consumer warps
constexpr int kConsumers = kWarps * 32;    // 384
constexpr int kThreads = kConsumers + 32;  // + the producer warp
constexpr int kDesc = 32;                  // ring descriptors (units in flight)
constexpr int kSmemBytes = 227 * 1024;
constexpr int kScratchBytes = 32 * 1024;   // x staging | attention scores / reduction
constexpr int kPartialBytes = 5 * 1024;    // per-slice row sums of a GEMV stage
constexpr int kMiscBytes = 2048;
constexpr int kRingBytes = kSmemBytes - kScratchBytes - kPartialBytes - kMiscBytes;
constexpr int kMaxSplitTokens = kScratchBytes / 16;  // attention: 16 B per token
constexpr int kTileBytes = 576;                      // 16 rows x 64 k: 512 B nibbles + 64 B scales
constexpr int kRunTokens = 64;                       // K / V tokens per bulk copy (at most)
constexpr unsigned long long kWaitNs = 2000000000ull;

static_assert(kRingBytes % 16 == 0, "ring alignment");

// ------------------------------------------------------------------ small helpers
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }

__device__ __forceinline__ bool mbar_wait_timed(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  unsigned long long t0 = 0;
  for (uint32_t i = 0;; i++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 255) == 255) {
      if (*abort_flag) return false;
      const unsigned long long t = gtimer();
      if (t0 == 0) t0 = t;
      else if (t - t0 > kWaitNs) return false;
    }
  }
}

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1, int c1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(c1), "r"(0), "r"(c1));
}

__device__ __forceinline__ unsigned long long argmax_key(uint16_t bits, int idx) {
  uint32_t u = (uint32_t)bits << 16;
  uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}

// logical row of position p (0..15) in row group rg
__host__ __device__ __forceinline__ int t16_row(int rowmap, int rg, int p, int n, int head_dim) {
  if (rowmap == SPARK_ROWS_PAIR_HALF) {
    const int per = head_dim >> 4, hd = rg / per, s = rg - hd * per;
    return hd * head_dim + (p < 8 ? 8 * s + p : (head_dim >> 1) + 8 * s + (p - 8));
  }
  if (rowmap == SPARK_ROWS_GATE_UP) return p < 8 ? 8 * rg + p : (n >> 1) + 8 * rg + (p - 8);
  return 16 * rg + p;
}

__host__ __device__ __forceinline__ int split_len(int64_t len, int splits) {
  const int64_t t = (len + splits - 1) / splits;
  return (int)((t + 15) / 16 * 16);
}

// number of units of a GEMV stage that CTA `cta` owns, and its first unit
__host__ __device__ __forceinline__ int local_units(const SparkStage& s, int cta, int ncta, int& u0) {
  u0 = (cta - s.rot + ncta) % ncta;
  return u0 < s.units ? (s.units - u0 + ncta - 1) / ncta : 0;
}

// attention task of CTA `cta`: kv head g and split j, or false
__host__ __device__ __forceinline__ bool attn_task(const SparkStage& s, int cta, int& g, int& j) {
  if (cta >= s.nkv * s.splits) return false;
  g = cta / s.splits;
  j = cta - g * s.splits;
  return true;
}

// ------------------------------------------------------------------ shared memory
struct Smem {
  unsigned char* ring;
  unsigned char* scratch;
  float* partial;
  unsigned long long* full;   // [kDesc] mbarriers
  unsigned long long* empty;  // [kDesc]
  uint32_t* desc_off;         // [kDesc]
  int* done;                  // [kDesc] finished tasks of the unit in the slot
  uint32_t* prod_start;       // [kDesc] producer bookkeeping
  uint32_t* prod_end;         // [kDesc]
  volatile int* abort_flag;
  int* flag;                  // [4] misc flags
  float* red;                 // [64] reductions
  unsigned long long* red64;  // [16]
  SparkStage* stage;          // consumers' copy of the current stage
};

__device__ __forceinline__ Smem carve(unsigned char* base) {
  Smem s;
  s.ring = base;
  s.scratch = base + kRingBytes;
  s.partial = reinterpret_cast<float*>(base + kRingBytes + kScratchBytes);
  unsigned char* m = base + kRingBytes + kScratchBytes + kPartialBytes;
  s.full = reinterpret_cast<unsigned long long*>(m);
  s.empty = s.full + kDesc;
  s.desc_off = reinterpret_cast<uint32_t*>(s.empty + kDesc);
  s.done = reinterpret_cast<int*>(s.desc_off + kDesc);
  s.prod_start = reinterpret_cast<uint32_t*>(s.done + kDesc);
  s.prod_end = s.prod_start + kDesc;
  s.abort_flag = reinterpret_cast<volatile int*>(s.prod_end + kDesc);
  s.flag = reinterpret_cast<int*>(s.prod_end + kDesc) + 4;
  s.red = reinterpret_cast<float*>(s.flag + 4);
  s.red64 = reinterpret_cast<unsigned long long*>(s.red + 64);
  s.stage = reinterpret_cast<SparkStage*>(s.red64 + 16);
  return s;
}
// 256 + 256 + 128 + 128 + 128 + 128 + 16 + 16 + 256 + 128 + 256 = 1696 <= kMiscBytes
static_assert(sizeof(SparkStage) == 256, "SparkStage layout");

struct StepParams {
  SparkStage inline_stage;   // the program when it has one stage (8-byte aligned)
  const SparkStage* stages;  // device program (nullptr: the single inline stage)
  int num_stages;
  SparkStepIO io;
};

__device__ __forceinline__ const SparkStage& stage_at(const StepParams& P, int i) {
  return P.stages ? P.stages[i] : P.inline_stage;
}

__device__ __forceinline__ void raise_abort(const StepParams& P, const Smem& s, int code) {
  *s.abort_flag = 1;
  atomicExch(P.io.counters + P.num_stages + 1, 1);
  if (P.io.error) atomicCAS(P.io.error, 0, code);
}

// ------------------------------------------------------------------ producer
struct Producer {
  const StepParams& P;
  const Smem& s;
  uint32_t seq = 0, tail = 0, head = 0;

  __device__ Producer(const StepParams& p, const Smem& sm) : P(p), s(sm) {}

  __device__ bool issue(const void* src, uint32_t bytes) {
    if (*s.abort_flag) return false;
    uint32_t a = head;
    if (a + bytes > (uint32_t)kRingBytes) a = 0;
    while (tail < seq) {
      bool must = seq - tail >= (uint32_t)kDesc;
      for (uint32_t u = tail; !must && u < seq; u++) {
        const uint32_t b0 = s.prod_start[u % kDesc], b1 = s.prod_end[u % kDesc];
        must = (a < b1) && (b0 < a + bytes);
      }
      if (!must) break;
      if (!mbar_wait_timed(smem_u32(s.empty + tail % kDesc), (tail / kDesc) & 1u, s.abort_flag)) {
        raise_abort(P, s, SPARK_ERR_LAUNCH);
        return false;
      }
      tail++;
    }
    const uint32_t slot = seq % kDesc;
    s.prod_start[slot] = a;
    s.prod_end[slot] = a + bytes;
    s.desc_off[slot] = a;
    head = a + bytes;
    const uint32_t bar = smem_u32(s.full + slot);
    mbar_expect_tx(bar, bytes);
    bulk_g2s(smem_u32(s.ring + a), src, bytes, bar);
    seq++;
    return true;
  }

  __device__ void run() {
    const int ncta = gridDim.x, cta = blockIdx.x;
    for (int i = 0; i < P.num_stages; i++) {
      const SparkStage& st = stage_at(P, i);
      if (st.kind == SPARK_STAGE_GEMV) {
        int u0;
        const int nl = local_units(st, cta, ncta, u0);
        const uint32_t ub = (uint32_t)(9 * (st.k / st.kp));
        for (int j = 0; j < nl; j++) {
          const unsigned char* src = static_cast<const unsigned char*>(st.w) + (size_t)(u0 + j * ncta) * ub;
          if (!issue(src, ub)) return drain();
        }
      } else {
        int g, j;
        if (!attn_task(st, cta, g, j)) continue;
        const int64_t len = st.pos[0] + 1;
        const int T = split_len(len, st.splits);
        if (T > kMaxSplitTokens) return drain();
        const int64_t t0 = (int64_t)j * T, t1 = t0 + T < len ? t0 + T : len;
        if (t1 <= t0) continue;
        const int64_t w0 = t0 / kRunTokens, nruns = (t1 - 1) / kRunTokens - w0 + 1;
        const int D = st.head_dim, bs = st.block_size, nkv = st.nkv;
        for (int side = 0; side < 2; side++) {
          const uint16_t* cache = static_cast<const uint16_t*>(side ? st.v_cache : st.k_cache);
          for (int64_t r = 0; r < nruns; r++) {
            const int64_t rs = (w0 + r) * kRunTokens > t0 ? (w0 + r) * kRunTokens : t0;
            const int64_t re = (w0 + r + 1) * kRunTokens < t1 ? (w0 + r + 1) * kRunTokens : t1;
            const int64_t page = st.block_table[rs / bs];
            const uint16_t* src = cache + ((page * nkv + g) * bs + (rs % bs)) * D;
            if (!issue(src, (uint32_t)((re - rs) * D * 2))) return drain();
          }
        }
      }
    }
    drain();
  }

  // every issued copy has landed before the CTA may exit
  __device__ void drain() {
    for (uint32_t u = tail; u < seq; u++) {
      if (!mbar_wait_timed(smem_u32(s.full + u % kDesc), (u / kDesc) & 1u, s.abort_flag)) {
        // abort raised elsewhere: still wait for the bytes in flight, bounded
        for (uint32_t v = u; v < seq; v++) {
          volatile int never = 0;
          mbar_wait_timed(smem_u32(s.full + v % kDesc), (v / kDesc) & 1u, &never);
        }
        return;
      }
    }
  }
};

// ------------------------------------------------------------------ consumers: x staging
// Block b of x becomes X_j = rint(x_j * 2^S), S = 13 - e (e = exponent of the block
// maximum), split into signed digits X = 256 h + l.  MMA B fragment of block b:
// entry e in 0..7 (lane & 7): e < 4 -> column 0 (h) with k = 4e.., e >= 4 -> column 1
// (l) with k = 4(e-4)..; .x holds k 0..15, .y holds k 16..31.  meta = (-8 sum X, sx).
__device__ __forceinline__ void stage_block13(const float (&v)[32], uint2* xfrag, int2* xmeta, int b) {
  float M = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; j++) M = fmaxf(M, fabsf(v[j]));
  int X[32];
  float sx = 1.0f;
  int sum = 0;
  if (M >= 7.888609052210118e-31f && M != __int_as_float(0x7f800000)) {
    const int e = (int)((__float_as_uint(M) >> 23) & 0xffu) - 127;
    const int S = 13 - e;
    const float sc = __uint_as_float((uint32_t)(S + 127) << 23);
#pragma unroll
    for (int j = 0; j < 32; j++) {
      X[j] = __float2int_rn(__fmul_rn(v[j], sc));
      sum += X[j];
    }
    sx = __uint_as_float((uint32_t)(127 - S) << 23);
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++) X[j] = 0;
  }
  uint32_t hw[8], lw[8];
#pragma unroll
  for (int w = 0; w < 8; w++) {
    uint32_t hh = 0, ll = 0;
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const int x = X[4 * w + t];
      const int l = ((x + 128) & 255) - 128;
      const int h = (x - l) >> 8;
      hh |= (uint32_t)(h & 0xff) << (8 * t);
      ll |= (uint32_t)(l & 0xff) << (8 * t);
    }
    hw[w] = hh;
    lw[w] = ll;
  }
#pragma unroll
  for (int c = 0; c < 4; c++) {
    xfrag[b * 8 + c] = make_uint2(hw[c], hw[4 + c]);
    xfrag[b * 8 + 4 + c] = make_uint2(lw[c], lw[4 + c]);
  }
  xmeta[b] = make_int2(-8 * sum, __float_as_int(sx));
}

// input element i of the stage's a operand (bf16 value as fp32)
__device__ __forceinline__ float a_elem(const SparkStage& st, const uint16_t* arow, int i) {
  if (st.pro == SPARK_PRO_PARTS) {
    const float* p = static_cast<const float*>(st.a);
    float v = __ldcg(p + i);
    for (int q = 1; q < st.a_parts; q++) v = __fadd_rn(v, __ldcg(p + (size_t)q * st.k + i));
    return bf2f(f2bf(v));
  }
  return bf2f(__ldcg(arow + i));
}

__device__ void stage_x(const SparkStage& st, const Smem& s, int tid) {
  const int k = st.k, nb = k >> 5;
  uint2* xfrag = reinterpret_cast<uint2*>(s.scratch);
  int2* xmeta = reinterpret_cast<int2*>(s.scratch + 64 * nb);
  float* slin = reinterpret_cast<float*>(s.scratch + 72 * nb);
  const uint16_t* arow = static_cast<const uint16_t*>(st.a);
  if (st.embed) arow = static_cast<const uint16_t*>(st.embed) + (size_t)__ldcg(st.token) * k;
  if (!st.norm) {
    for (int b = tid; b < nb; b += kConsumers) {
      float v[32];
#pragma unroll 8
      for (int j = 0; j < 32; j++) v[j] = a_elem(st, arow, b * 32 + j);
      stage_block13(v, xfrag, xmeta, b);
    }
    return;
  }
  const uint16_t* bb = static_cast<const uint16_t*>(st.b);
  uint16_t* res = (blockIdx.x == 0) ? static_cast<uint16_t*>(st.res_out) : nullptr;
  for (int i = tid; i < k; i += kConsumers) {
    float v = a_elem(st, arow, i);
    if (bb) v = __fadd_rn(v, bf2f(__ldcg(bb + i)));
    slin[i] = v;
    if (res) res[i] = f2bf(v);
  }
  consumer_bar();
  if (tid < 32) {
    float acc = 0.0f;
    for (int i = tid; i < k; i += 32) acc = __fadd_rn(acc, __fmul_rn(slin[i], slin[i]));
    acc = butterfly_sum<32>(acc);
    if (tid == 0) s.red[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(acc, st.inv_k), st.eps)));
  }
  consumer_bar();
  const float inv = s.red[0];
  const uint16_t* gm = static_cast<const uint16_t*>(st.gamma);
  for (int b = tid; b < nb; b += kConsumers) {
    float v[32];
#pragma unroll 8
    for (int j = 0; j < 32; j++) v[j] = bf2f(f2bf(__fmul_rn(__fmul_rn(slin[b * 32 + j], inv), bf2f(gm[b * 32 + j]))));
    stage_block13(v, xfrag, xmeta, b);
  }
}

// ------------------------------------------------------------------ consumers: GEMV
// one (unit, slice) task: lanes 4g hold the slice sums of positions g and g + 8
__device__ __forceinline__ void gemv_task(const SparkStage& st, const Smem& s, uint32_t ubase, int kpi, int sl,
                                          int lane, float& acc0, float& acc1) {
  const int Kp = st.k / st.kp, tiles = Kp >> 6, tps = tiles / st.ks;
  const uint2* xfrag = reinterpret_cast<const uint2*>(s.scratch);
  const int2* xmeta = reinterpret_cast<const int2*>(s.scratch + 64 * (st.k >> 5));
  const int gb0 = kpi * (Kp >> 5);
  const uint32_t m = 0x0f0f0f0fu;
  acc0 = 0.0f;
  acc1 = 0.0f;
  const int t_end = (sl + 1) * tps;
#pragma unroll 2
  for (int t = sl * tps; t < t_end; t++) {
    const uint32_t tb = ubase + (uint32_t)t * kTileBytes;
    uint4 w;
    uint2 dd;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                 : "r"(tb + lane * 16));
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(dd.x), "=r"(dd.y) : "r"(tb + 512 + (lane >> 2) * 8));
#pragma unroll
    for (int half = 0; half < 2; half++) {
      const int gb = gb0 + 2 * t + half;
      const uint2 bx = xfrag[gb * 8 + (lane & 7)];
      const int2 meta = xmeta[gb];
      const uint32_t wg = half ? w.z : w.x, wg8 = half ? w.w : w.y;
      int d[4];
      mma_u8s8(d, wg & m, wg8 & m, (wg >> 4) & m, (wg8 >> 4) & m, bx.x, bx.y, meta.x);
      const int p0 = d[0] * 256 + d[1], p1 = d[2] * 256 + d[3];
      const uint32_t hv = half ? dd.y : dd.x;
      const float sx = __int_as_float(meta.y);
      acc0 = __fmaf_rn(__fmul_rn(h2f((uint16_t)(hv & 0xffffu)), sx), (float)p0, acc0);
      acc1 = __fmaf_rn(__fmul_rn(h2f((uint16_t)(hv >> 16)), sx), (float)p1, acc1);
    }
  }
}

__device__ __forceinline__ uint16_t bf16r(float v) { return f2bf(v); }

// epilogue of one row pair (positions g and g + 8 of unit u)
__device__ __forceinline__ void gemv_epilogue(const SparkStage& st, int u, int g, float v0, float v1,
                                              unsigned long long& best) {
  const int rg = u / st.kp, kpi = u - rg * st.kp;
  const int r0 = t16_row(st.rowmap, rg, g, st.n, st.head_dim);
  const int r1 = t16_row(st.rowmap, rg, g + 8, st.n, st.head_dim);
  switch (st.epi) {
    case SPARK_EPI_BF16: {
      uint16_t* y = static_cast<uint16_t*>(st.out);
      y[r0] = bf16r(v0);
      y[r1] = bf16r(v1);
      break;
    }
    case SPARK_EPI_PARTS: {
      float* y = static_cast<float*>(st.out) + (size_t)kpi * st.n;
      y[r0] = v0;
      y[r1] = v1;
      break;
    }
    case SPARK_EPI_SILU_MUL: {
      const float gf = bf2f(f2bf(v0)), uf = bf2f(f2bf(v1));
      const float act = bf2f(f2bf(__fdiv_rn(gf, __fadd_rn(1.0f, spark_exp(-gf)))));
      static_cast<uint16_t*>(st.out)[r0] = f2bf(__fmul_rn(act, uf));
      break;
    }
    case SPARK_EPI_ARGMAX: {
      const uint16_t b0 = f2bf(v0), b1 = f2bf(v1);
      if (st.out) {
        static_cast<uint16_t*>(st.out)[r0] = b0;
        static_cast<uint16_t*>(st.out)[r1] = b1;
      }
      const unsigned long long k0 = argmax_key(b0, r0), k1 = argmax_key(b1, r1);
      const unsigned long long k = k0 > k1 ? k0 : k1;
      best = k > best ? k : best;
      break;
    }
    default: {  // SPARK_EPI_ROPE_KV
      const int D = st.head_dim, half = D >> 1;
      const int hd = r0 / D, i = r0 - hd * D;
      const int64_t pos = __ldcg(st.pos);
      float a = bf2f(f2bf(v0)), b = bf2f(f2bf(v1));
      if (hd < st.nq + st.nkv) {
        const uint16_t* cs = static_cast<const uint16_t*>(st.cos_sin) + (size_t)pos * D;
        const float c = bf2f(cs[i]), sn = bf2f(cs[i + half]);
        const float u2 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
        const float w2 = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, sn));
        a = u2;
        b = w2;
      }
      const uint16_t ua = f2bf(a), ub = f2bf(b);
      if (hd < st.nq) {
        uint16_t* q = static_cast<uint16_t*>(st.q) + (size_t)hd * D;
        q[i] = ua;
        q[i + half] = ub;
      } else {
        const int isv = hd >= st.nq + st.nkv;
        const int hk = hd - st.nq - isv * st.nkv;
        const int64_t blk = pos / st.block_size, off = pos - blk * st.block_size;
        const int64_t slot_blk = st.block_table[blk];
        uint16_t* cache = static_cast<uint16_t*>(isv ? st.v_cache : st.k_cache);
        uint16_t* dst = cache + ((slot_blk * st.nkv + hk) * st.block_size + off) * D;
        dst[i] = ua;
        dst[i + half] = ub;
        uint16_t* kn = static_cast<uint16_t*>(st.kv_new) + ((size_t)isv * st.nkv + hk) * D;
        kn[i] = ua;
        kn[i + half] = ub;
      }
      break;
    }
  }
}

__device__ __forceinline__ bool wait_unit(const Smem& s, uint32_t seq) {
  return mbar_wait_timed(smem_u32(s.full + seq % kDesc), (seq / kDesc) & 1u, s.abort_flag);
}

// the task that completes a unit releases its ring bytes
__device__ __forceinline__ void finish_task(const Smem& s, uint32_t seq, int tasks, int lane) {
  __syncwarp();
  if (lane == 0) {
    const uint32_t slot = seq % kDesc;
    if (atomicAdd(s.done + slot, 1) == tasks - 1) {
      s.done[slot] = 0;
      mbar_arrive(smem_u32(s.empty + slot));
    }
  }
}

__device__ bool gemv_stage(const StepParams& P, const SparkStage& st, const Smem& s, uint32_t& seq_base, int tid) {
  const int ncta = gridDim.x, cta = blockIdx.x, warp = tid >> 5, lane = tid & 31;
  int u0;
  const int nl = local_units(st, cta, ncta, u0);
  if (nl > 0 || (cta == 0 && st.res_out)) stage_x(st, s, tid);
  consumer_bar();
  const int ks = st.ks;
  for (int t = warp; t < nl * ks; t += kWarps) {
    const int j = t / ks, sl = t - j * ks;
    const uint32_t seq = seq_base + j;
    if (!wait_unit(s, seq)) {  // abort: skip the work, keep the barriers
      raise_abort(P, s, SPARK_ERR_LAUNCH);
      continue;
    }
    const int u = u0 + j * ncta;
    float acc0, acc1;
    gemv_task(st, s, smem_u32(s.ring) + s.desc_off[seq % kDesc], u % st.kp, sl, lane, acc0, acc1);
    if ((lane & 3) == 0) {
      s.partial[(j * ks + sl) * 16 + (lane >> 2)] = acc0;
      s.partial[(j * ks + sl) * 16 + (lane >> 2) + 8] = acc1;
    }
    finish_task(s, seq, ks, lane);
  }
  consumer_bar();
  unsigned long long best = 0ull;
  for (int f = tid; f < nl * 8; f += kConsumers) {
    const int j = f >> 3, g = f & 7;
    const float* pr = s.partial + j * ks * 16;
    float v0 = pr[g], v1 = pr[g + 8];
    for (int q = 1; q < ks; q++) {
      v0 = __fadd_rn(v0, pr[q * 16 + g]);
      v1 = __fadd_rn(v1, pr[q * 16 + g + 8]);
    }
    gemv_epilogue(st, u0 + j * ncta, g, v0, v1, best);
  }
  if (st.epi == SPARK_EPI_ARGMAX) {
#pragma unroll
    for (int off = 16; off >= 1; off /= 2) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
      best = o > best ? o : best;
    }
    if (lane == 0) s.red64[warp] = best;
    consumer_bar();
    if (tid == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < kWarps; w++) m = s.red64[w] > m ? s.red64[w] : m;
      if (m) atomicMax(st.key, m);
    }
  }
  seq_base += nl;
  return true;
}

// ------------------------------------------------------------------ consumers: attention
// Task (kv head g, split j): tokens [t0, t1) of the context pos + 1, T = split_len.
// Scores: 8 lanes per token (lane jj owns dims 8jj..8jj+7, 64+8jj..64+8jj+7; even /
// odd positions in two fma chains, butterfly 4,2,1); rec[i] = 4 scores (fp32).  Then
// max, p = exp(s - m) in place, l per head in the 32-lane order, P = bf16(p) in place.
// PV: 16-token chunk c is summed by warp c % 12 (lane owns dims 4 lane .. +3 of all 4
// heads); the 12 warp sums are added in warp order.  The last split of a head to
// finish combines all splits of its 4 q heads into attn_out.
__device__ bool attn_stage(const StepParams& P, const SparkStage& st, const Smem& s, uint32_t& seq_base, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  int g, j;
  if (!attn_task(st, blockIdx.x, g, j)) return true;
  const int D = 128, nq = st.nq, S = st.splits;
  const int64_t pos = __ldcg(st.pos), len = pos + 1;
  const int T = split_len(len, S);
  if (T > kMaxSplitTokens) {
    if (tid == 0) raise_abort(P, s, SPARK_ERR_TOO_LARGE);
    return false;
  }
  const int64_t t0 = (int64_t)j * T, t1 = t0 + T < len ? t0 + T : len;
  const int n = t1 > t0 ? (int)(t1 - t0) : 0;
  float* part_o = st.part_o;
  float* part_lse = st.part_lse;
  const uint16_t* kv_new = static_cast<const uint16_t*>(st.kv_new);
  float4* rec = reinterpret_cast<float4*>(s.scratch);
  if (n == 0) {
    for (int o = tid; o < 4 * D; o += kConsumers) part_o[((size_t)j * nq + 4 * g) * D + o] = 0.0f;
    if (tid < 4) part_lse[(size_t)j * nq + 4 * g + tid] = __int_as_float(0xff800000);
  } else {
    const int64_t w0 = t0 / kRunTokens;
    const int nruns = (int)((t1 - 1) / kRunTokens - w0 + 1);
    const int nch = (n + 15) >> 4;
    const int jj = lane & 7, grp = lane >> 3;
    // q: 4 heads x 16 dims of this lane
    float qf[4][16];
    {
      const uint16_t* q = static_cast<const uint16_t*>(st.q) + (size_t)4 * g * D;
#pragma unroll
      for (int h = 0; h < 4; h++)
#pragma unroll
        for (int m = 0; m < 16; m++) qf[h][m] = bf2f(__ldcg(q + h * D + (m < 8 ? 8 * jj + m : 64 + 8 * jj + m - 8)));
    }
    auto run_of = [&](int64_t ts, int64_t& rs, int64_t& re) {
      const int64_t r = ts / kRunTokens - w0;
      rs = (w0 + r) * kRunTokens > t0 ? (w0 + r) * kRunTokens : t0;
      re = (w0 + r + 1) * kRunTokens < t1 ? (w0 + r + 1) * kRunTokens : t1;
      return (int)r;
    };
    // ---- scores
    for (int c = warp; c < nch; c += kWarps) {
      const int64_t ts = t0 + 16 * c;
      int64_t rs, re;
      const int r = run_of(ts, rs, re);
      const uint32_t seq = seq_base + r;
      if (!wait_unit(s, seq)) {  // abort: skip the work, keep the barriers
        raise_abort(P, s, SPARK_ERR_LAUNCH);
        continue;
      }
      const unsigned char* rowbase = s.ring + s.desc_off[seq % kDesc] + (ts - rs) * 256;
#pragma unroll 1
      for (int step4 = 0; step4 < 4; step4++) {
        const int i = 16 * c + 4 * step4 + grp;
        const bool valid = i < n;
        uint4 k0 = make_uint4(0, 0, 0, 0), k1 = k0;
        if (valid) {
          const int64_t t = t0 + i;
          if (t == pos) {
            const uint16_t* kr = kv_new + (size_t)g * D;
            k0 = __ldcg(reinterpret_cast<const uint4*>(kr + 8 * jj));
            k1 = __ldcg(reinterpret_cast<const uint4*>(kr + 64 + 8 * jj));
          } else {
            const unsigned char* kr = rowbase + (4 * step4 + grp) * 256;
            k0 = *reinterpret_cast<const uint4*>(kr + 16 * jj);
            k1 = *reinterpret_cast<const uint4*>(kr + 128 + 16 * jj);
          }
        }
        const uint32_t kw[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
        float sc[4];
#pragma unroll
        for (int h = 0; h < 4; h++) {
          float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
          for (int m = 0; m < 8; m++) {
            a0 = __fmaf_rn(qf[h][2 * m], bf_lo(kw[m]), a0);
            a1 = __fmaf_rn(qf[h][2 * m + 1], bf_hi(kw[m]), a1);
          }
          float v = __fadd_rn(a0, a1);
          v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
          v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
          v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
          sc[h] = __fmul_rn(v, st.scale);
        }
        if (valid && jj == 0) rec[i] = make_float4(sc[0], sc[1], sc[2], sc[3]);
      }
      finish_task(s, seq, (int)((re - rs + 15) >> 4), lane);
    }
    consumer_bar();
    // ---- max (exact in any order)
    {
      float m4[4] = {__int_as_float(0xff800000), __int_as_float(0xff800000), __int_as_float(0xff800000),
                     __int_as_float(0xff800000)};
      for (int i = tid; i < n; i += kConsumers) {
        const float4 r4 = rec[i];
        m4[0] = r4.x > m4[0] ? r4.x : m4[0];
        m4[1] = r4.y > m4[1] ? r4.y : m4[1];
        m4[2] = r4.z > m4[2] ? r4.z : m4[2];
        m4[3] = r4.w > m4[3] ? r4.w : m4[3];
      }
#pragma unroll
      for (int h = 0; h < 4; h++) {
        float v = m4[h];
#pragma unroll
        for (int off = 16; off >= 1; off /= 2) {
          const float o = __shfl_xor_sync(0xffffffffu, v, off);
          v = o > v ? o : v;
        }
        if (lane == 0) s.red[warp * 4 + h] = v;
      }
    }
    consumer_bar();
    float mh[4];
#pragma unroll
    for (int h = 0; h < 4; h++) {
      float v = s.red[h];
      for (int w = 1; w < kWarps; w++) v = s.red[w * 4 + h] > v ? s.red[w * 4 + h] : v;
      mh[h] = v;
    }
    for (int i = tid; i < n; i += kConsumers) {
      const float4 r4 = rec[i];
      rec[i] = make_float4(spark_exp(__fsub_rn(r4.x, mh[0])), spark_exp(__fsub_rn(r4.y, mh[1])),
                           spark_exp(__fsub_rn(r4.z, mh[2])), spark_exp(__fsub_rn(r4.w, mh[3])));
    }
    consumer_bar();
    if (warp < 4) {
      const float* pf = reinterpret_cast<const float*>(rec);
      float acc = 0.0f;
      for (int i = lane; i < n; i += 32) acc = __fadd_rn(acc, pf[4 * i + warp]);
      acc = butterfly_sum<32>(acc);
      if (lane == 0) s.red[48 + warp] = acc;
    }
    consumer_bar();
    for (int i = tid; i < n; i += kConsumers) {
      const float4 r4 = rec[i];
      uint2 pb;
      pb.x = (uint32_t)f2bf(r4.x) | ((uint32_t)f2bf(r4.y) << 16);
      pb.y = (uint32_t)f2bf(r4.z) | ((uint32_t)f2bf(r4.w) << 16);
      *reinterpret_cast<uint2*>(rec + i) = pb;
    }
    consumer_bar();
    // ---- PV
    float acc[4][4];
#pragma unroll
    for (int h = 0; h < 4; h++)
#pragma unroll
      for (int d = 0; d < 4; d++) acc[h][d] = 0.0f;
    for (int c = warp; c < nch; c += kWarps) {
      const int64_t ts = t0 + 16 * c;
      int64_t rs, re;
      const int r = run_of(ts, rs, re);
      const uint32_t seq = seq_base + nruns + r;
      if (!wait_unit(s, seq)) {  // abort: skip the work, keep the barriers
        raise_abort(P, s, SPARK_ERR_LAUNCH);
        continue;
      }
      const unsigned char* rowbase = s.ring + s.desc_off[seq % kDesc] + (ts - rs) * 256;
      const int cnt = n - 16 * c < 16 ? n - 16 * c : 16;
      for (int tt = 0; tt < cnt; tt++) {
        const int i = 16 * c + tt;
        const uint2 pb = *reinterpret_cast<const uint2*>(rec + i);
        const float p4[4] = {bf_lo(pb.x), bf_hi(pb.x), bf_lo(pb.y), bf_hi(pb.y)};
        uint2 vv;
        if (t0 + i == pos) {
          vv = __ldcg(reinterpret_cast<const uint2*>(kv_new + ((size_t)st.nkv + g) * D + 4 * lane));
        } else {
          vv = *reinterpret_cast<const uint2*>(rowbase + tt * 256 + 8 * lane);
        }
        const float v4[4] = {bf_lo(vv.x), bf_hi(vv.x), bf_lo(vv.y), bf_hi(vv.y)};
#pragma unroll
        for (int h = 0; h < 4; h++)
#pragma unroll
          for (int d = 0; d < 4; d++) acc[h][d] = __fmaf_rn(p4[h], v4[d], acc[h][d]);
      }
      finish_task(s, seq, (int)((re - rs + 15) >> 4), lane);
    }
    const float lh = s.red[48 + (tid & 3)];  // read before the scratch is reused
    consumer_bar();
    float* red_o = reinterpret_cast<float*>(s.scratch);
#pragma unroll
    for (int h = 0; h < 4; h++)
      *reinterpret_cast<float4*>(red_o + (warp * 4 + h) * D + 4 * lane) =
          make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    consumer_bar();
    for (int o = tid; o < 4 * D; o += kConsumers) {
      const int h = o >> 7, d = o & 127;
      float v = red_o[h * D + d];
      for (int w = 1; w < kWarps; w++) v = __fadd_rn(v, red_o[(w * 4 + h) * D + d]);
      part_o[((size_t)j * nq + 4 * g + h) * D + d] = __fdiv_rn(v, s.red[48 + h]);
    }
    if (tid < 4) part_lse[(size_t)j * nq + 4 * g + tid] = __fadd_rn(spark_log(lh), mh[tid]);
    seq_base += 2 * nruns;
  }
  // ---- the last split of head g combines
  consumer_bar();
  if (tid == 0) {
    __threadfence();
    s.flag[0] = atomicAdd(st.head_counters + g, 1) == S - 1;
  }
  consumer_bar();
  if (!s.flag[0]) return true;
  __threadfence();
  float* wgt = reinterpret_cast<float*>(s.scratch);  // [4][S] weights, then [4] empty flags
  if (tid < 4) {
    const int h = tid;
    float mx = __int_as_float(0xff800000);
    for (int sp = 0; sp < S; sp++) {
      const float v = __ldcg(part_lse + (size_t)sp * nq + 4 * g + h);
      mx = v > mx ? v : mx;
    }
    float den = 0.0f;
    for (int sp = 0; sp < S; sp++) {
      const float v = __ldcg(part_lse + (size_t)sp * nq + 4 * g + h);
      const float w = (v == __int_as_float(0xff800000)) ? 0.0f : spark_exp(__fsub_rn(v, mx));
      wgt[h * S + sp] = w;
      den = __fadd_rn(den, w);
    }
    for (int sp = 0; sp < S; sp++) wgt[h * S + sp] = __fdiv_rn(wgt[h * S + sp], den);
    s.red[56 + h] = (mx == __int_as_float(0xff800000)) ? 1.0f : 0.0f;
  }
  consumer_bar();
  uint16_t* out = static_cast<uint16_t*>(st.attn_out);
  for (int o = tid; o < 4 * D; o += kConsumers) {
    const int h = o >> 7, d = o & 127;
    float a = 0.0f;
    if (s.red[56 + h] == 0.0f) {
      for (int sp = 0; sp < S; sp++) {
        if (__ldcg(part_lse + (size_t)sp * nq + 4 * g + h) == __int_as_float(0xff800000)) continue;
        a = __fadd_rn(a, __fmul_rn(wgt[h * S + sp], __ldcg(part_o + ((size_t)sp * nq + 4 * g + h) * D + d)));
      }
    }
    out[(size_t)(4 * g + h) * D + d] = f2bf(a);
  }
  if (tid == 0) st.head_counters[g] = 0;
  return true;
}

// ------------------------------------------------------------------ the kernel
__device__ __forceinline__ bool wait_stage(const StepParams& P, const Smem& s, int idx) {
  const int* ctr = P.io.counters + idx;
  const int target = (int)gridDim.x;
  if (ld_acquire(ctr) >= target) return true;
  const unsigned long long t0 = gtimer();
  for (;;) {
    __nanosleep(20);
    if (ld_acquire(ctr) >= target) return true;
    if (ld_acquire(P.io.counters + P.num_stages + 1)) return false;
    if (gtimer() - t0 > kWaitNs) return false;
  }
}

__global__ void __launch_bounds__(kThreads, 1) step_kernel(const StepParams P) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const Smem s = carve(smem_raw);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < kDesc; i++) {
      mbar_init(smem_u32(s.full + i), 1);
      mbar_init(smem_u32(s.empty + i), 1);
      s.done[i] = 0;
    }
    *s.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid >= kConsumers) {
    if (tid == kConsumers) {
      Producer pr(P, s);
      pr.run();
    }
    return;
  }
  uint32_t seq_base = 0;
  for (int i = 0; i < P.num_stages; i++) {
    if (tid < 32)  // 8-byte pieces: the inline stage in the launch parameters is only 8-byte aligned
      reinterpret_cast<unsigned long long*>(s.stage)[tid] =
          reinterpret_cast<const unsigned long long*>(&stage_at(P, i))[tid];
    if (tid == 0) {
      const int w = stage_at(P, i).wait;
      int stop = *s.abort_flag;
      if (!stop && w >= 0 && !wait_stage(P, s, w)) {
        raise_abort(P, s, SPARK_ERR_LAUNCH);
        stop = 1;
      }
      s.flag[1] = stop;
    }
    consumer_bar();
    if (s.flag[1]) return;  // uniform: every consumer reads the same flag
    const SparkStage& st = *s.stage;
    // both stage functions keep every consumer on the same barriers; a stage that
    // fails returns false in all threads (attention: a split longer than the scratch)
    const bool ok = st.kind == SPARK_STAGE_GEMV ? gemv_stage(P, st, s, seq_base, tid)
                                                : attn_stage(P, st, s, seq_base, tid);
    consumer_bar();
    if (!ok) return;
    if (tid == 0 && !*s.abort_flag) {
      __threadfence();
      atomicAdd(P.io.counters + i, 1);
    }
  }
  // ---- the last CTA to finish turns the argmax into a token and resets the counters
  if (tid == 0 && !*s.abort_flag) {
    __threadfence();
    const int done = atomicAdd(P.io.counters + P.num_stages, 1);
    if (done == (int)gridDim.x - 1) {
      __threadfence();
      const SparkStepIO& io = P.io;
      if (io.key) {
        const unsigned long long k = atomicAdd(io.key, 0ull);
        const int32_t tok = (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
        if (io.token_out) io.token_out[0] = tok;
        if (io.token_log) io.token_log[io.step ? io.step[0] : 0] = tok;
        *io.key = 0ull;
      }
      if (io.step) io.step[0] += 1;
      if (io.pos) io.pos[0] += 1;
      for (int i = 0; i <= P.num_stages; i++) P.io.counters[i] = 0;
      __threadfence();
    }
  }
}

// ------------------------------------------------------------------ T16 packing
__global__ void t16_pack_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ d, int n, int k, int kp,
                                int rowmap, int aux, uint8_t* __restrict__ out) {
  const int Kp = k / kp, tiles = Kp >> 6;
  const size_t unit_bytes = (size_t)9 * Kp;
  const size_t total = (size_t)(n >> 4) * kp * tiles * 32;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int L = (int)(i & 31);
    const size_t tt = i >> 5;
    const int t = (int)(tt % tiles);
    const int u = (int)(tt / tiles);
    const int rg = u / kp, kpi = u - rg * kp;
    const int g = L >> 2, c = L & 3;
    const int ra = t16_row(rowmap, rg, g, n, aux), rb = t16_row(rowmap, rg, g + 8, n, aux);
    const int b0 = kpi * (Kp >> 5) + 2 * t;
    const uint8_t* qa = qs + (size_t)ra * (k >> 1) + (size_t)b0 * 16 + 4 * c;
    const uint8_t* qb = qs + (size_t)rb * (k >> 1) + (size_t)b0 * 16 + 4 * c;
    uint4 v;
    v.x = *reinterpret_cast<const uint32_t*>(qa);
    v.y = *reinterpret_cast<const uint32_t*>(qb);
    v.z = *reinterpret_cast<const uint32_t*>(qa + 16);
    v.w = *reinterpret_cast<const uint32_t*>(qb + 16);
    uint8_t* tile = out + (size_t)u * unit_bytes + (size_t)t * kTileBytes;
    *reinterpret_cast<uint4*>(tile + 16 * L) = v;
    if (c == 0) {
      const size_t nb = (size_t)(k >> 5);
      uint2 dv;
      dv.x = (uint32_t)d[(size_t)ra * nb + b0] | ((uint32_t)d[(size_t)rb * nb + b0] << 16);
      dv.y = (uint32_t)d[(size_t)ra * nb + b0 + 1] | ((uint32_t)d[(size_t)rb * nb + b0 + 1] << 16);
      *reinterpret_cast<uint2*>(tile + 512 + 8 * g) = dv;
    }
  }
}

}  // namespace step
}  // namespace spark
