// step_kernel.cuh -- the persistent decode-step kernel (one cooperative launch per
// decode step, one CTA per SM).
//
// A launch runs a program of stages (SparkStage, include/spark_b200.h): GEMV stages
// over Q4_0 weights in the T16 layout, and split-KV attention stages.  Every CTA has
// a producer warp and 11 consumer warps:
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

constexpr int kWarps = 11;                 // consumer warps (12 warps per CTA keep 168 registers)
constexpr int kConsumers = kWarps * 32;    // 352
constexpr int kThreads = kConsumers + 32;  // + the producer warp
constexpr int kDesc = 16;                  // ring descriptors (units in flight)
constexpr int kMaxSlices = 4;              // GEMV slices per unit (per-slot slice sums)
constexpr int kTraceSlots = 24;            // trace stamps per stage
constexpr int kSmemBytes = 227 * 1024;
constexpr int kScratchBytes = 40 * 1024;   // x staging | attention scores / reduction / combine
constexpr int kPartialBytes = kDesc * kMaxSlices * 16 * 4;  // slice sums per ring slot
constexpr int kMiscBytes = 2048;
constexpr int kRingBytes = kSmemBytes - kScratchBytes - kPartialBytes - kMiscBytes;
constexpr int kMaxSplitTokens = 1344;  // attention: 24 B of scratch per token (scores + P)
constexpr int kTileBytes = 576;                      // 16 rows x 64 k: 512 B nibbles + 64 B scales
constexpr int kRunTokens = 64;                       // K / V tokens per bulk copy (at most)
constexpr unsigned long long kWaitNs = 2000000000ull;

static_assert(kRingBytes % 16 == 0, "ring alignment");

// Shared-memory budget of a batch-NB program (NB = 1: the constants above).  A batch
// stage stages NB input vectors: NB x 72 B per 32-element block of digits / meta, and for
// an RMSNorm prologue the NB pre-norm vectors in fp32 (4 k NB bytes, reused by the digits)
// plus gamma; its slice sums are NB x 16 per slice (ks <= 2); the per-sequence launch
// constants (position, cache row, RoPE row) sit in the misc area.
template <int NB>
struct Layout {
  static constexpr int scratch = NB == 1 ? kScratchBytes : (NB == 2 ? 40 * 1024 : (NB == 4 ? 48 * 1024 : 88 * 1024));
  static constexpr int slices = NB == 1 ? kMaxSlices : 2;
  static constexpr int partial = kDesc * slices * 16 * 4 * NB;
  static constexpr int misc = NB == 1 ? kMiscBytes : 4608;
  static constexpr int ring = kSmemBytes - scratch - partial - misc;
  static_assert(ring % 16 == 0 && ring >= 96 * 1024, "ring");
};
static_assert(Layout<1>::ring == kRingBytes, "one-sequence layout");

// ------------------------------------------------------------------ small helpers
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// cycle checkpoint (clock64) for the optional trace: slot k of the stage's stamps
__device__ __forceinline__ void cstamp(unsigned long long* tr, int k) {
  if (tr) tr[k] = (unsigned long long)clock64();
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
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

// float(P) without an int-to-float conversion: for |P| < 2^22 the bits of P + kMagic
// are the fp32 1.5 * 2^23 + P, exactly; subtracting 1.5 * 2^23 leaves P exactly.
// |P| <= 32 * 8 * 16320 < 2^22 for the staged digits (|X| <= 16320).
constexpr int kMagic = 0x4B400000;
constexpr float kMagicF = 12582912.0f;

__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1, int c1) {
  asm(
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

// t16_row with the Spark qkv layout: aux = head_dim | rotary_dim << 16 for
// SPARK_ROWS_PAIR_HALF (rotary_dim 0: head_dim): per head, the rotary pairs (i, i + r/2)
// (r/16 units), then dims r.. in plain runs of 16; rows past the last whole head (the
// gate rows) plain.  Equal to t16_row when rotary_dim is 0 and n is whole heads.
__host__ __device__ __forceinline__ int t16_row_x(int rowmap, int rg, int p, int n, int aux) {
  if (rowmap != SPARK_ROWS_PAIR_HALF) return t16_row(rowmap, rg, p, n, aux);
  const int head_dim = aux & 0xffff, r = (aux >> 16) ? (aux >> 16) : head_dim;
  const int per = head_dim >> 4, hd = rg / per, s = rg - hd * per;
  if ((hd + 1) * head_dim > n) return hd * head_dim + 16 * s + p;
  const int npair = r >> 4;
  if (s < npair) return hd * head_dim + (p < 8 ? 8 * s + p : (r >> 1) + 8 * s + (p - 8));
  return hd * head_dim + r + 16 * (s - npair) + p;
}

__host__ __device__ __forceinline__ int split_len(int64_t len, int splits) {
  const int64_t t = (len + splits - 1) / splits;
  return (int)((t + 15) / 16 * 16);
}

// bytes of a Q6_K unit in the T6 layout: 16 rows x kp_cols columns (6.5625 bits each)
__host__ __device__ __forceinline__ uint32_t t6_unit_bytes(int kp_cols) { return (uint32_t)(105 * kp_cols / 8); }

// number of units of a GEMV stage that CTA `cta` owns, its first unit and the stride
// between its units.  SPARK_PRO_ATTN (o_proj fused behind attention, kp = kv heads):
// CTA c < kp * splits holds kv head c / splits's combined output, so it takes K part
// c / splits of the row groups c % splits, c % splits + splits, ...; other stages rotate
// their units over all CTAs (first unit `rot` on CTA 0).
__host__ __device__ __forceinline__ int local_units(const SparkStage& s, int cta, int ncta, int& u0, int& ustride) {
  if (s.pro == SPARK_PRO_ATTN) {
    const int grp = cta / s.splits, jj = cta - grp * s.splits, rgs = s.n >> 4;
    u0 = jj * s.kp + grp;
    ustride = s.splits * s.kp;
    return grp < s.kp && jj < rgs ? (rgs - jj + s.splits - 1) / s.splits : 0;
  }
  u0 = (cta - s.rot + ncta) % ncta;
  ustride = ncta;
  return u0 < s.units ? (s.units - u0 + ncta - 1) / ncta : 0;
}

// ------------------------------------------------------------------ shared memory
struct Smem {
  unsigned char* ring;
  unsigned char* scratch;
  float* partial;
  unsigned long long* full;   // [kDesc] mbarriers
  unsigned long long* empty;  // [kDesc]
  uint32_t* desc_off;         // [kDesc]
  uint32_t* desc_seq;         // [kDesc] sequence number of the copy last issued into the slot
  int* done;                  // [kDesc] finished tasks of the unit in the slot
  uint32_t* prod_start;       // [kDesc] producer bookkeeping
  uint32_t* prod_end;         // [kDesc]
  volatile int* abort_flag;
  int* flag;                  // [4] misc flags
  float* red;                 // [64] reductions
  unsigned long long* red64;  // [16]
  SparkStage* stage;          // consumers' copy of the current stage
  long long* misc64;          // [4] per-stage values (position, cache row offset)
  uint16_t* rope_cs;          // [256] cos | sin row of the position (RoPE stages); batch: [NB][128]
  long long* bpos;            // batch: [NB] positions
  long long* bkvoff;          // batch: [NB] paged-cache element offsets of the decoded tokens
};

template <int NB>
__device__ __forceinline__ Smem carve(unsigned char* base) {
  using L = Layout<NB>;
  Smem s;
  s.ring = base;
  s.scratch = base + L::ring;
  s.partial = reinterpret_cast<float*>(base + L::ring + L::scratch);
  unsigned char* m = base + L::ring + L::scratch + L::partial;
  s.full = reinterpret_cast<unsigned long long*>(m);
  s.empty = s.full + kDesc;
  s.desc_off = reinterpret_cast<uint32_t*>(s.empty + kDesc);
  s.desc_seq = s.desc_off + kDesc;
  s.done = reinterpret_cast<int*>(s.desc_seq + kDesc);
  s.prod_start = reinterpret_cast<uint32_t*>(s.done + kDesc);
  s.prod_end = s.prod_start + kDesc;
  s.abort_flag = reinterpret_cast<volatile int*>(s.prod_end + kDesc);
  s.flag = reinterpret_cast<int*>(s.prod_end + kDesc) + 4;
  s.red = reinterpret_cast<float*>(s.flag + 4);
  s.red64 = reinterpret_cast<unsigned long long*>(s.red + 64);
  s.stage = reinterpret_cast<SparkStage*>(s.red64 + 16 * NB);
  s.misc64 = reinterpret_cast<long long*>(s.stage + 1);
  s.rope_cs = reinterpret_cast<uint16_t*>(s.misc64 + 4);
  s.bpos = reinterpret_cast<long long*>(s.rope_cs + (NB == 1 ? 256 : 128 * NB));
  s.bkvoff = s.bpos + NB;
  return s;
}
// full 128 + empty 128 + desc_off / desc_seq / done / prod_start / prod_end 5 x 64 + abort / flag 32 +
// red 256 + red64 128 NB + stage 288 + misc64 32 + rope_cs 512 (batch: 256 NB) + bpos / bkvoff 16 NB:
// 1824 (NB = 1) <= kMiscBytes, 4480 (NB = 8) <= Layout<8>::misc
static_assert(sizeof(SparkStage) == 288, "SparkStage layout");
constexpr int kStageWords = (int)sizeof(SparkStage) / 8;

struct StepParams {
  SparkStage inline_stage;   // the program when it has one stage (8-byte aligned)
  const SparkStage* stages;  // device program (nullptr: the single inline stage)
  int num_stages;
  SparkStepIO io;
};

__device__ __forceinline__ const SparkStage& stage_at(const StepParams& P, int i) {
  return P.stages ? P.stages[i] : P.inline_stage;
}

// ------------------------------------------------------------------ tensor parallelism
// The same exchange-window address as mapped for rank p.
template <typename T>
__device__ __forceinline__ T* peer_addr(const SparkStepIO& io, int p, T* local) {
  const unsigned long long off =
      (unsigned long long)reinterpret_cast<uintptr_t>(local) - (unsigned long long)reinterpret_cast<uintptr_t>(io.window);
  return reinterpret_cast<T*>((uintptr_t)(io.peer_windows[p] + off));
}

// Counter value at which stage `st` is complete in this launch.  Single GPU: counters
// are zeroed between launches, so CTAs; tensor parallel: never reset, so
// contributors x (launch + 1), compared wrap-safe.
__device__ __forceinline__ int stage_target(const SparkStepIO& io, const SparkStage& st, int ncta, long long launch) {
  if (io.tp_size <= 1) return ncta;
  const int contrib = st.xchg ? ncta * io.tp_size : ncta;
  return (int)((unsigned)contrib * (unsigned)(launch + 1));
}
__device__ __forceinline__ bool reached(int v, int target) { return (int)((unsigned)v - (unsigned)target) >= 0; }

__device__ __forceinline__ void raise_abort(const StepParams& P, const Smem& s, int code) {
  *s.abort_flag = 1;
  atomicExch(P.io.counters + P.num_stages + 1, 1);
  if (P.io.error) atomicCAS(P.io.error, 0, code);
}

// ------------------------------------------------------------------ producer
// NB: the program's batch (ring size; attention tasks of NB sequences)
template <int NB>
struct Producer {
  const StepParams& P;
  const Smem& s;
  uint32_t seq = 0, tail = 0, head = 0, tail_off = 0;

  __device__ Producer(const StepParams& p, const Smem& sm) : P(p), s(sm) {}

  // The ring is a FIFO of byte ranges: outstanding units occupy [tail_off, head)
  // circularly, tail_off being the start of the oldest unit not yet released.
  __device__ bool issue(const void* src, uint32_t bytes) {
    if (*s.abort_flag) return false;
    uint32_t a = head;
    if (a + bytes > (uint32_t)Layout<NB>::ring) a = 0;
    while (tail < seq) {
      if (seq - tail < (uint32_t)kDesc) {
        const uint32_t t = tail_off;
        const bool ok = t < head ? (a >= head || a + bytes <= t)    // free: [head, R) and [0, t)
                                 : (t > head && a == head && a + bytes <= t);  // free: [head, t)
        if (ok) break;
      }
      if (!mbar_wait_timed(smem_u32(s.empty + tail % kDesc), (tail / kDesc) & 1u, s.abort_flag)) {
        raise_abort(P, s, SPARK_ERR_LAUNCH);
        return false;
      }
      tail++;
      tail_off = tail < seq ? s.prod_start[tail % kDesc] : head;
    }
    const uint32_t slot = seq % kDesc;
    if (tail == seq) tail_off = a;
    s.prod_start[slot] = a;
    s.desc_off[slot] = a;
    *reinterpret_cast<volatile uint32_t*>(s.desc_seq + slot) = seq;  // (ordered before the arrive below)
    head = a + bytes;
    const uint32_t bar = smem_u32(s.full + slot);
    mbar_expect_tx(bar, bytes);
    bulk_g2s(smem_u32(s.ring + a), src, bytes, bar);
    seq++;
    return true;
  }

  // Multi: attention tasks may outnumber the CTAs (several per CTA); Spark: sliding
  // window attention stages
  template <bool Multi, bool Spark>
  __device__ void run() {
    const int ncta = gridDim.x, cta = blockIdx.x;
    for (int i = 0; i < P.num_stages; i++) {
      const SparkStage& st = stage_at(P, i);
      if (P.io.trace) P.io.trace[((size_t)cta * P.num_stages + i) * kTraceSlots + 3] = gtimer();
      if (st.kind == SPARK_STAGE_GEMV || st.kind == SPARK_STAGE_GEMV_Q6) {
        int u0, ustride;
        const int nl = local_units(st, cta, ncta, u0, ustride);
        const uint32_t ub = (uint32_t)(st.kind == SPARK_STAGE_GEMV_Q6 ? t6_unit_bytes(st.k / st.kp) : 9 * (st.k / st.kp));
        for (int j = 0; j < nl; j++) {
          const unsigned char* src = static_cast<const unsigned char*>(st.w) + (size_t)(u0 + j * ustride) * ub;
          if (!issue(src, ub)) return drain();
        }
      } else {
        // this CTA's tasks (sequence b, kv head g, split j) in the consumers' order: K then V
        // runs each
        const int S = st.splits, ntask = NB * st.nkv * S;
        // K then V runs of task t; false: aborted
        auto task = [&](int t) -> bool {
          const int b = NB == 1 ? 0 : t / (st.nkv * S), tb = t - b * st.nkv * S;
          const int g = tb / S, j = tb - g * S;
          const int64_t len = st.pos[b] + 1;
          // (Spark sliding window: splits from the window start rounded down to 16)
          const int64_t start = (Spark && st.window > 0 && len > st.window ? len - st.window : 0) & ~(int64_t)15;
          const int T = split_len(len - start, S);
          if (T > kMaxSplitTokens) return false;
          const int64_t t0 = start + (int64_t)j * T, t1 = t0 + T < len ? t0 + T : len;
          if (t1 <= t0) return true;
          const int64_t w0 = t0 / kRunTokens, nruns = (t1 - 1) / kRunTokens - w0 + 1;
          const int D = st.head_dim, bs = st.block_size, nkv = st.nkv;
          const int32_t* table = st.block_table + (NB == 1 ? 0 : (size_t)b * st.bt_stride);
          for (int side = 0; side < 2; side++) {
            const uint16_t* cache = static_cast<const uint16_t*>(side ? st.v_cache : st.k_cache);
            for (int64_t r = 0; r < nruns; r++) {
              const int64_t rs = (w0 + r) * kRunTokens > t0 ? (w0 + r) * kRunTokens : t0;
              const int64_t re = (w0 + r + 1) * kRunTokens < t1 ? (w0 + r + 1) * kRunTokens : t1;
              const int64_t page = table[rs / bs];
              const uint16_t* src = cache + ((page * nkv + g) * bs + (rs % bs)) * D;
              if (!issue(src, (uint32_t)((re - rs) * D * 2))) return false;
            }
          }
          return true;
        };
        if constexpr (Multi) {
          for (int t = cta; t < ntask; t += ncta)
            if (!task(t)) return drain();
        } else if (cta < ntask && !task(cta)) {
          return drain();
        }
      }
      if (P.io.trace) P.io.trace[((size_t)cta * P.num_stages + i) * kTraceSlots + 10] = gtimer();
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
// (l) with k = 4(e-4)..; word 0 holds k 0..15, word 1 holds k 16..31.
// meta = (-8 sum X, sx).  Four consecutive threads stage one block, 8 elements each.
constexpr int kStageGroups = 4;  // 8-element groups per consumer thread (k <= 12288)
constexpr int kMaxParts = 8;  // parts summed by a PARTS prologue (K parts x TP ranks)
constexpr int kPartsBatch = 4;  // parts loaded per L2 round trip
constexpr int kTaggedBatch = 2;  // tagged exchange parts read per round trip

__device__ __forceinline__ void lds_u32x4(uint32_t addr, uint4& v) {
  asm("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
}
__device__ __forceinline__ void lds_u32x2(uint32_t addr, uint2& v) {
  asm("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
}

__device__ __forceinline__ void unpack8(const uint4 u, float (&v)[8]) {
  v[0] = bf_lo(u.x); v[1] = bf_hi(u.x); v[2] = bf_lo(u.y); v[3] = bf_hi(u.y);
  v[4] = bf_lo(u.z); v[5] = bf_hi(u.z); v[6] = bf_lo(u.w); v[7] = bf_hi(u.w);
}

// x -> bf16 (round to nearest even) -> fp32 in one conversion instruction; matches f2bf
// for every non-NaN input
__device__ __forceinline__ float bf16_round(float x) {
  uint16_t h;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(x));
  return __uint_as_float((uint32_t)h << 16);
}

// two floats -> packed bf16 pair (lo in the low half), round to nearest even
__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// low bytes of four ints -> one word (byte t from x_t)
__device__ __forceinline__ uint32_t pack_bytes(int x0, int x1, int x2, int x3) {
  return __byte_perm(__byte_perm((uint32_t)x0, (uint32_t)x1, 0x0040), __byte_perm((uint32_t)x2, (uint32_t)x3, 0x0040),
                     0x5410);
}

// stage the 8 elements of group g (block g / 4, elements 8 (g % 4) ..); the 4 lanes of a
// block are consecutive lanes of one warp and all execute this (valid or not)
// xmeta2 (nullable, Q6_K stages): (-32 sum of X over elements 0..15, over 16..31)
// bs: records between consecutive blocks (a batch of NB sequences interleaves its
// sequences' records: block b of sequence q at record b NB + q)
__device__ __forceinline__ void stage_group(const float (&v)[8], bool valid, int g, uint32_t* xfrag32, int2* xmeta,
                                            int2* xmeta2 = nullptr, int bs = 1) {
  float M = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; j++) M = fmaxf(M, fabsf(v[j]));
  M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 1));
  M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 2));
  const bool live = M >= 7.888609052210118e-31f && M != __int_as_float(0x7f800000);
  const int e = (int)((__float_as_uint(M) >> 23) & 0xffu) - 127;
  const int S = 13 - e;
  const float sc = live ? __uint_as_float((uint32_t)(S + 127) << 23) : 0.0f;
  int X[8], sum = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    X[j] = live ? __float2int_rn(__fmul_rn(v[j], sc)) : 0;
    sum += X[j];
  }
  sum += __shfl_xor_sync(0xffffffffu, sum, 1);  // lanes 0, 1: X 0..15; lanes 2, 3: X 16..31
  const int half_other = __shfl_xor_sync(0xffffffffu, sum, 2);
  if (valid && xmeta2 && (g & 3) == 0) xmeta2[g >> 2] = make_int2(-32 * sum, -32 * half_other);
  sum += half_other;
  if (!valid) return;
  const int b = g >> 2, c = g & 3;
#pragma unroll
  for (int w = 0; w < 2; w++) {
    int hv[4], lv[4];
#pragma unroll
    for (int t = 0; t < 4; t++) {  // X = 256 h + l, l in [-128, 127]
      hv[t] = (X[4 * w + t] + 128) >> 8;
      lv[t] = X[4 * w + t] - 256 * hv[t];
    }
    const uint32_t hh = pack_bytes(hv[0], hv[1], hv[2], hv[3]);
    const uint32_t ll = pack_bytes(lv[0], lv[1], lv[2], lv[3]);
    const int word = 2 * c + w;  // k = 4 word .. 4 word + 3
    xfrag32[(b * bs * 8 + (word & 3)) * 2 + (word >> 2)] = hh;
    xfrag32[(b * bs * 8 + 4 + (word & 3)) * 2 + (word >> 2)] = ll;
  }
  // meta.x = -8 sum X + kMagic: the MMA's column-1 accumulator input, so that
  // 256 D0 + D1 = P + kMagic is P as the low mantissa bits of 1.5 * 2^23 (|P| < 2^22)
  if (c == 0)
    xmeta[b * bs] =
        make_int2(-8 * sum + kMagic, __float_as_int(live ? __uint_as_float((uint32_t)(127 - S) << 23) : 1.0f));
}

// group handled by slot gi of this CTA (out-of-range slots stay out of range)
__device__ __forceinline__ int stage_grp(int gi, int ngrp, int rot) {
  if (gi >= ngrp) return gi;
  const int g = gi + rot;
  return g >= ngrp ? g - ngrp : g;
}

// Sum, in part order, the 8 elements of group g of a_parts tagged parts (uint64 words:
// fp32 bits | tag << 32, part q at tp + q k) once every word carries this launch's tag:
// each batch of parts is re-read until it does (bounded like every wait).  Only the
// tensor-parallel kernel instantiations carry it, so its registers stay out of the  false: the wait ran out or the launch
// aborted.
__device__ __forceinline__ bool tagged_parts_sum(const unsigned long long* tp, int a_parts, int k, int g, uint32_t tag,
                                              volatile int* abort_flag, float4& p0, float4& p1) {
  bool first = true, ok = true;
  for (int q2 = 0; q2 < a_parts; q2 += kTaggedBatch) {
    unsigned long long wv[kTaggedBatch][8];
    unsigned long long t0 = 0;
    for (uint32_t it = 0;; it++) {
      bool ready = true;
#pragma unroll
      for (int q = 0; q < kTaggedBatch; q++) {
        if (q2 + q < a_parts) {
          const unsigned long long* src = tp + (size_t)(q2 + q) * k + 8 * g;
#pragma unroll
          for (int j = 0; j < 8; j += 2)
            asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];"
                         : "=l"(wv[q][j]), "=l"(wv[q][j + 1])
                         : "l"(src + j)
                         : "memory");
#pragma unroll
          for (int j = 0; j < 8; j++) ready = ready && (uint32_t)(wv[q][j] >> 32) == tag;
        }
      }
      if (ready) break;
      if ((it & 15) == 15) {
        const unsigned long long t = gtimer();
        if (t0 == 0) t0 = t;
        if (*abort_flag || t - t0 > kWaitNs) {
          ok = false;
          break;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kTaggedBatch; q++) {
      if (q2 + q < a_parts) {
        const float4 a0 = make_float4(__uint_as_float((uint32_t)wv[q][0]), __uint_as_float((uint32_t)wv[q][1]),
                                      __uint_as_float((uint32_t)wv[q][2]), __uint_as_float((uint32_t)wv[q][3]));
        const float4 a1 = make_float4(__uint_as_float((uint32_t)wv[q][4]), __uint_as_float((uint32_t)wv[q][5]),
                                      __uint_as_float((uint32_t)wv[q][6]), __uint_as_float((uint32_t)wv[q][7]));
        if (first) {
          p0 = a0;
          p1 = a1;
          first = false;
        } else {
          p0 = make_float4(__fadd_rn(p0.x, a0.x), __fadd_rn(p0.y, a0.y), __fadd_rn(p0.z, a0.z), __fadd_rn(p0.w, a0.w));
          p1 = make_float4(__fadd_rn(p1.x, a1.x), __fadd_rn(p1.y, a1.y), __fadd_rn(p1.z, a1.z), __fadd_rn(p1.w, a1.w));
        }
      }
    }
    if (!ok) break;
  }
  return ok;
}

template <bool Q6, bool TP>
__device__ __forceinline__ void stage_x(const StepParams& P, const SparkStage& st, const Smem& s, int tid,
                                        unsigned long long* tr, int x0,
                                        int kx) {
  const int k = st.k, nb = kx >> 5, ngrp = kx >> 3;
  uint32_t* xfrag32 = reinterpret_cast<uint32_t*>(s.scratch);
  int2* xmeta = reinterpret_cast<int2*>(s.scratch + 64 * nb);
  // Q6_K stages also need the half-block sums: after the norm area (squares, gamma)
  int2* xmeta2 = (Q6 && st.kind == SPARK_STAGE_GEMV_Q6) ? reinterpret_cast<int2*>(s.scratch + 72 * nb + 6 * k) : nullptr;
  float* sq = reinterpret_cast<float*>(s.scratch + 72 * nb);
  const uint16_t* arow = static_cast<const uint16_t*>(st.a) + x0;
  if (st.embed) arow = static_cast<const uint16_t*>(st.embed) + (size_t)__ldcg(st.token) * k + x0;
  const float* parts = static_cast<const float*>(st.a) + x0;
  const uint16_t* bb = st.b ? static_cast<const uint16_t*>(st.b) + x0 : nullptr;
  const uint16_t* gm = reinterpret_cast<const uint16_t*>(s.scratch + 72 * nb + 4 * k);  // prefetched gamma
  float v[kStageGroups][8];
  uint4 gv[kStageGroups];
  // Every CTA reads the whole input vector at the same moment: start each CTA at a
  // different block (a multiple of 4 groups keeps a block's 4 lanes together) so the
  // requests spread over the L2 slices instead of queueing on the same lines.
  const int rot = 4 * (int)((blockIdx.x * 37u) % (unsigned)(ngrp >> 2));
  // all loads first: one L2 round trip
  if (st.pro == SPARK_PRO_PARTS || st.pro == SPARK_PRO_PARTS_TAGGED) {
    // parts in flight in batches, then summed in part order.  A PARTS input has at most
    // one 8-element group per thread (k <= kConsumers * 8, the host checks): slot 0.
    const int g = stage_grp(tid, ngrp, rot);
#pragma unroll
    for (int r = 1; r < kStageGroups; r++)
#pragma unroll
      for (int j = 0; j < 8; j++) v[r][j] = 0.0f;
    if (g < ngrp) {
      uint4 bv = make_uint4(0, 0, 0, 0);
      if (st.norm) {
        if (bb) bv = __ldcg(reinterpret_cast<const uint4*>(bb + 8 * g));
        gv[0] = *reinterpret_cast<const uint4*>(gm + 8 * g);
      }
      float4 p0 = make_float4(0.f, 0.f, 0.f, 0.f), p1 = p0;
      if (TP && st.pro == SPARK_PRO_PARTS_TAGGED) {
        if (!tagged_parts_sum(static_cast<const unsigned long long*>(st.a) + x0, st.a_parts, k, g,
                              (uint32_t)(s.misc64[2] + 1), s.abort_flag, p0, p1))
          raise_abort(P, s, SPARK_ERR_LAUNCH);
      } else
#pragma unroll
      for (int q4 = 0; q4 < kMaxParts; q4 += kPartsBatch) {  // kPartsBatch parts per round trip
        if (q4 < st.a_parts) {
          float4 q0[kPartsBatch], q1[kPartsBatch];
#pragma unroll
          for (int q = 0; q < kPartsBatch; q++) {
            if (q4 + q < st.a_parts) {
              q0[q] = __ldcg(reinterpret_cast<const float4*>(parts + (size_t)(q4 + q) * k + 8 * g));
              q1[q] = __ldcg(reinterpret_cast<const float4*>(parts + (size_t)(q4 + q) * k + 8 * g + 4));
            }
          }
#pragma unroll
          for (int q = 0; q < kPartsBatch; q++) {
            if (q4 + q == 0) {
              p0 = q0[0];
              p1 = q1[0];
            } else if (q4 + q < st.a_parts) {
              p0 = make_float4(__fadd_rn(p0.x, q0[q].x), __fadd_rn(p0.y, q0[q].y), __fadd_rn(p0.z, q0[q].z),
                               __fadd_rn(p0.w, q0[q].w));
              p1 = make_float4(__fadd_rn(p1.x, q1[q].x), __fadd_rn(p1.y, q1[q].y), __fadd_rn(p1.z, q1[q].z),
                               __fadd_rn(p1.w, q1[q].w));
            }
          }
        }
      }
      const float t8[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
      for (int j = 0; j < 8; j++) v[0][j] = bf16_round(t8[j]);
      if (st.norm && bb) {
        float w8[8];
        unpack8(bv, w8);
#pragma unroll
        for (int j = 0; j < 8; j++) v[0][j] = __fadd_rn(v[0][j], w8[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) v[0][j] = 0.0f;
    }
  } else {
#pragma unroll
  for (int r = 0; r < kStageGroups; r++) {
    const int g = stage_grp(tid + r * kConsumers, ngrp, rot);
    if (g < ngrp) {
      uint4 bv = make_uint4(0, 0, 0, 0);
      if (st.norm) {
        if (bb) bv = __ldcg(reinterpret_cast<const uint4*>(bb + 8 * g));  // with the first loads
        gv[r] = *reinterpret_cast<const uint4*>(gm + 8 * g);
      }
      unpack8(__ldcg(reinterpret_cast<const uint4*>(arow + 8 * g)), v[r]);
      if (st.norm && bb) {
        float w8[8];
        unpack8(bv, w8);
#pragma unroll
        for (int j = 0; j < 8; j++) v[r][j] = __fadd_rn(v[r][j], w8[j]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) v[r][j] = 0.0f;
    }
  }
  }
  if (tr) tr[6] = gtimer();
  if (st.norm) {
    uint16_t* res = (blockIdx.x == 0) ? static_cast<uint16_t*>(st.res_out) : nullptr;
#pragma unroll
    for (int r = 0; r < kStageGroups; r++) {
      const int g = stage_grp(tid + r * kConsumers, ngrp, rot);
      if (g < ngrp) {
#pragma unroll
        for (int j = 0; j < 8; j++) sq[8 * g + j] = __fmul_rn(v[r][j], v[r][j]);
        if (res) {
          uint4 o;
          o.x = bf16x2(v[r][0], v[r][1]);
          o.y = bf16x2(v[r][2], v[r][3]);
          o.z = bf16x2(v[r][4], v[r][5]);
          o.w = bf16x2(v[r][6], v[r][7]);
          *reinterpret_cast<uint4*>(res + 8 * g) = o;
        }
      }
    }
    consumer_bar();
    if (tid < 32) {  // canonical order: lane l sums s_i^2, i = l mod 32, ascending
      float acc = 0.0f;
      int i = tid;
      for (; i + 15 * 32 < k; i += 16 * 32) {  // 16 loads in flight, then the ordered adds
        float q16[16];
#pragma unroll
        for (int q = 0; q < 16; q++) q16[q] = sq[i + 32 * q];
#pragma unroll
        for (int q = 0; q < 16; q++) acc = __fadd_rn(acc, q16[q]);
      }
      for (; i < k; i += 32) acc = __fadd_rn(acc, sq[i]);
      acc = butterfly_sum<32>(acc);
      if (tid == 0) s.red[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(acc, st.inv_k), st.eps)));
    }
    consumer_bar();
    if (tr) tr[7] = gtimer();
    const float inv = s.red[0];
#pragma unroll
    for (int r = 0; r < kStageGroups; r++) {
      if (r * kConsumers >= ngrp) break;
      float g8[8];
      unpack8(gv[r], g8);
#pragma unroll
      for (int j = 0; j < 8; j++) v[r][j] = bf16_round(__fmul_rn(__fmul_rn(v[r][j], inv), g8[j]));
    }
  }
#pragma unroll
  for (int r = 0; r < kStageGroups; r++) {
    const int g = stage_grp(tid + r * kConsumers, ngrp, rot);
    if (r * kConsumers < ngrp) stage_group(v[r], g < ngrp, g, xfrag32, xmeta, xmeta2);
  }
}


// ------------------------------------------------------------------ batch x staging
// A batch-NB stage stages the NB sequences' input vectors with the arithmetic of stage_x,
// sequence by sequence the same (the RMSNorm's canonical order included), so each
// sequence's digits equal those of its one-sequence launch.  Work items are (sequence q,
// 8-element group g), item q ngrp + g, spread over the consumer threads from a rotated
// start as in stage_x.  Block b of sequence q lands at record b NB + q (stage_group's
// block stride), so the 4 blocks x NB sequences of a block group are one contiguous run.
// Norm stages keep the pre-norm values in fp32 in the scratch ([NB][k], the digits reuse
// it afterwards); warp q sums sequence q's squares.
constexpr int kBatchItems = 8;  // items per thread (NB k / 8 <= 8 x 352: k <= 2816 at NB = 8)

// the pre-norm values of item (q, g): the bf16 input (or the embedding row of token[q]),
// plus the residual b of a norm stage
__device__ __forceinline__ void batch_load_bf16(const SparkStage& st, int q, int g, int x0, float (&v)[8]) {
  const int k = st.k;
  const uint16_t* arow = st.embed ? static_cast<const uint16_t*>(st.embed) + (size_t)__ldcg(st.token + q) * k
                                  : static_cast<const uint16_t*>(st.a) + (size_t)q * k;
  unpack8(__ldcg(reinterpret_cast<const uint4*>(arow + x0 + 8 * g)), v);
  if (st.norm && st.b) {
    float w8[8];
    unpack8(__ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(st.b) + (size_t)q * k + x0 + 8 * g)),
            w8);
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __fadd_rn(v[j], w8[j]);
  }
}

// ... of a SPARK_PRO_PARTS norm stage: bf16 of the part sum (part order), plus b
__device__ __forceinline__ void batch_load_parts(const SparkStage& st, int q, int g, float (&v)[8]) {
  const int k = st.k;
  const float* parts = static_cast<const float*>(st.a) + (size_t)q * st.a_parts * k + 8 * g;
  uint4 bv = make_uint4(0u, 0u, 0u, 0u);
  if (st.b) bv = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(st.b) + (size_t)q * k + 8 * g));
  float4 p0 = __ldcg(reinterpret_cast<const float4*>(parts));
  float4 p1 = __ldcg(reinterpret_cast<const float4*>(parts + 4));
#pragma unroll 1
  for (int q4 = 1; q4 < st.a_parts; q4 += kPartsBatch) {
    float4 a0[kPartsBatch], a1[kPartsBatch];
#pragma unroll
    for (int i = 0; i < kPartsBatch; i++) {
      if (q4 + i < st.a_parts) {
        a0[i] = __ldcg(reinterpret_cast<const float4*>(parts + (size_t)(q4 + i) * k));
        a1[i] = __ldcg(reinterpret_cast<const float4*>(parts + (size_t)(q4 + i) * k + 4));
      }
    }
#pragma unroll
    for (int i = 0; i < kPartsBatch; i++) {
      if (q4 + i < st.a_parts) {
        p0 = make_float4(__fadd_rn(p0.x, a0[i].x), __fadd_rn(p0.y, a0[i].y), __fadd_rn(p0.z, a0[i].z),
                         __fadd_rn(p0.w, a0[i].w));
        p1 = make_float4(__fadd_rn(p1.x, a1[i].x), __fadd_rn(p1.y, a1[i].y), __fadd_rn(p1.z, a1[i].z),
                         __fadd_rn(p1.w, a1[i].w));
      }
    }
  }
  const float t8[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] = bf16_round(t8[j]);
  if (st.b) {
    float w8[8];
    unpack8(bv, w8);
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __fadd_rn(v[j], w8[j]);
  }
}

// Norm stages: the pre-norm values of the thread's items, IR items' loads per L2 round
// trip, into the fp32 buffer (and the residual output, CTA 0)
template <int IR, bool Parts>
__device__ __forceinline__ void batch_prenorm(const SparkStage& st, int tid, int nitem, int ngrp, int rot, float* vbuf,
                                              uint16_t* res) {
  const int k = st.k;
#pragma unroll 1
  for (int r0 = 0; r0 * kConsumers < nitem; r0 += IR) {
    float v[IR][8];
#pragma unroll
    for (int r = 0; r < IR; r++) {
      const int it = stage_grp(tid + (r0 + r) * kConsumers, nitem, rot);
      if (it < nitem) {
        const int q = it / ngrp;
        if constexpr (Parts)
          batch_load_parts(st, q, it - q * ngrp, v[r]);
        else
          batch_load_bf16(st, q, it - q * ngrp, 0, v[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < IR; r++) {
      const int it = stage_grp(tid + (r0 + r) * kConsumers, nitem, rot);
      if (it < nitem) {
        const int q = it / ngrp, g = it - q * ngrp;
        float4* dst = reinterpret_cast<float4*>(vbuf + (size_t)q * k + 8 * g);
        dst[0] = make_float4(v[r][0], v[r][1], v[r][2], v[r][3]);
        dst[1] = make_float4(v[r][4], v[r][5], v[r][6], v[r][7]);
        if (res) {
          uint4 o;
          o.x = bf16x2(v[r][0], v[r][1]);
          o.y = bf16x2(v[r][2], v[r][3]);
          o.z = bf16x2(v[r][4], v[r][5]);
          o.w = bf16x2(v[r][6], v[r][7]);
          *reinterpret_cast<uint4*>(res + (size_t)q * k + 8 * g) = o;
        }
      }
    }
  }
}

template <int NB>
__device__ __forceinline__ void stage_x_batch(const SparkStage& st, const Smem& s, int tid, unsigned long long* tr,
                                              int x0, int kx) {
  const int k = st.k, nb = kx >> 5, ngrp = kx >> 3, nitem = NB * ngrp;
  uint32_t* xfrag32 = reinterpret_cast<uint32_t*>(s.scratch);
  int2* xmeta = reinterpret_cast<int2*>(s.scratch + 64 * nb * NB);
  const int rot = 4 * (int)((blockIdx.x * 37u) % (unsigned)(nitem >> 2));
  if (!st.norm) {  // load and stage, kBatchItems / 2 items per L2 round trip
#pragma unroll 1
    for (int r0 = 0; r0 * kConsumers < nitem; r0 += kBatchItems / 2) {
      float v[kBatchItems / 2][8];
#pragma unroll
      for (int r = 0; r < kBatchItems / 2; r++) {
        const int it = stage_grp(tid + (r0 + r) * kConsumers, nitem, rot);
        if (it < nitem) {
          const int q = it / ngrp;
          batch_load_bf16(st, q, it - q * ngrp, x0, v[r]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++) v[r][j] = 0.0f;
        }
      }
#pragma unroll
      for (int r = 0; r < kBatchItems / 2; r++) {
        if ((r0 + r) * kConsumers < nitem) {
          const int it = stage_grp(tid + (r0 + r) * kConsumers, nitem, rot);
          const int q = it < nitem ? it / ngrp : 0;
          stage_group(v[r], it < nitem, it - q * ngrp, xfrag32 + 16 * q, xmeta + q, nullptr, NB);
        }
      }
    }
    if (tr) tr[6] = tr[7] = gtimer();
    return;
  }
  float* vbuf = reinterpret_cast<float*>(s.scratch);  // [NB][k] (norm stages stage the whole k)
  const uint16_t* gm = reinterpret_cast<const uint16_t*>(s.scratch + 4 * k * NB);  // prefetched gamma
  uint16_t* res = (blockIdx.x == 0) ? static_cast<uint16_t*>(st.res_out) : nullptr;
  if (st.pro == SPARK_PRO_PARTS)
    batch_prenorm<1, true>(st, tid, nitem, ngrp, rot, vbuf, res);
  else
    batch_prenorm<4, false>(st, tid, nitem, ngrp, rot, vbuf, res);
  if (tr) tr[6] = gtimer();
  consumer_bar();
  if (tid < 32 * NB) {  // warp q: sequence q's canonical sum (lane l: s_i^2, i = l mod 32, ascending)
    const float* sv = vbuf + (size_t)(tid >> 5) * k;
    float acc = 0.0f;
    int i = tid & 31;
    for (; i + 15 * 32 < k; i += 16 * 32) {
      float q16[16];
#pragma unroll
      for (int q = 0; q < 16; q++) q16[q] = sv[i + 32 * q];
#pragma unroll
      for (int q = 0; q < 16; q++) acc = __fadd_rn(acc, __fmul_rn(q16[q], q16[q]));
    }
    for (; i < k; i += 32) acc = __fadd_rn(acc, __fmul_rn(sv[i], sv[i]));
    acc = butterfly_sum<32>(acc);
    if ((tid & 31) == 0) s.red[tid >> 5] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(acc, st.inv_k), st.eps)));
  }
  consumer_bar();
  if (tr) tr[7] = gtimer();
  // normalized values as packed bf16 (the scratch is rewritten by the digits below)
  uint4 yq[kBatchItems];
#pragma unroll
  for (int r = 0; r < kBatchItems; r++) {
    const int it = stage_grp(tid + r * kConsumers, nitem, rot);
    if (r * kConsumers < nitem && it < nitem) {
      const int q = it / ngrp, g = it - q * ngrp;
      const float inv = s.red[q];
      const float4 a0 = *reinterpret_cast<const float4*>(vbuf + (size_t)q * k + 8 * g);
      const float4 a1 = *reinterpret_cast<const float4*>(vbuf + (size_t)q * k + 8 * g + 4);
      float g8[8];
      unpack8(*reinterpret_cast<const uint4*>(gm + 8 * g), g8);
      const float t8[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float y[8];
#pragma unroll
      for (int j = 0; j < 8; j++) y[j] = __fmul_rn(__fmul_rn(t8[j], inv), g8[j]);
      yq[r] = make_uint4(bf16x2(y[0], y[1]), bf16x2(y[2], y[3]), bf16x2(y[4], y[5]), bf16x2(y[6], y[7]));
    } else {
      yq[r] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  consumer_bar();
#pragma unroll
  for (int r = 0; r < kBatchItems; r++) {
    if (r * kConsumers < nitem) {
      const int it = stage_grp(tid + r * kConsumers, nitem, rot);
      const int q = it < nitem ? it / ngrp : 0;
      float y[8];
      unpack8(yq[r], y);
      stage_group(y, it < nitem, it - q * ngrp, xfrag32 + 16 * q, xmeta + q, nullptr, NB);
    }
  }
}

// ------------------------------------------------------------------ consumers: GEMV
// one (unit, slice) task: lanes 4g hold the slice sums of positions g and g + 8 as a
// packed pair.  Tiles are processed 4 at a time (8 blocks: all shared-memory loads,
// then the 8 MMAs, then the fma chain in block order), then one at a time.
__device__ __forceinline__ unsigned long long f2pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long fmul2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long fadd2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Integer MMA with the accumulator as input and output (D = A B + D).
__device__ __forceinline__ void mma_u8s8_acc(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// A group = 4 consecutive Q4_0 blocks of a 16-row unit (2 tiles).  Its 4 MMAs run as one
// accumulator chain: MMA j multiplies block j's nibbles by B columns 2j / 2j + 1 = block
// j's h / l digits (every other column zero: lane L supplies column L / 4 = the entry of
// block L / 8, masked to MMA L / 8), so at the end lane (g, c) holds block c's two digit
// sums for rows g and g + 8 -- every lane has a block to scale, not one lane in four.
// The accumulator input carries each block's -8 sum X + kMagic in its l column (the
// meta of block c, loaded by lane c), so 256 D_h + D_l = P + kMagic as before.  Per
// lane: acc = fma(fp32(d) * sx, P, acc) for its block, i.e. chain c of the slice takes
// blocks c, c + 4, c + 8, ... in ascending order.
struct GemvLane {
  uint32_t bmask[4];  // ~0 for MMA L / 8, else 0
};

// NG groups: all shared-memory loads, then the 4 chain steps of every group (the groups'
// chains interleaved), then the fma chain in group order
template <int NG>
__device__ __forceinline__ void gemv_groups(uint32_t& a_adr, uint32_t& d_adr, uint32_t& b_adr, uint32_t& m_adr,
                                            const GemvLane& gl, unsigned long long& acc) {
  const uint32_t m = 0x0f0f0f0fu;
  uint4 A[NG][2];
  uint2 B[NG], Mt[NG];
  uint32_t Ds[NG];
#pragma unroll
  for (int i = 0; i < NG; i++) {
    lds_u32x4(a_adr + i * 2 * kTileBytes, A[i][0]);
    lds_u32x4(a_adr + i * 2 * kTileBytes + kTileBytes, A[i][1]);
    lds_u32x2(b_adr + i * 256, B[i]);
    lds_u32x2(m_adr + i * 32, Mt[i]);
    asm("ld.shared.u32 %0, [%1];" : "=r"(Ds[i]) : "r"(d_adr + i * 2 * kTileBytes));
  }
  int D[NG][4];
#pragma unroll
  for (int i = 0; i < NG; i++) {
    D[i][0] = 0;
    D[i][1] = (int)Mt[i].x;
    D[i][2] = 0;
    D[i][3] = (int)Mt[i].x;
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
#pragma unroll
    for (int i = 0; i < NG; i++) {
      const uint4& a = A[i][j >> 1];
      const uint32_t w0 = (j & 1) ? a.z : a.x, w1 = (j & 1) ? a.w : a.y;
      mma_u8s8_acc(D[i], w0 & m, w1 & m, (w0 >> 4) & m, (w1 >> 4) & m, B[i].x & gl.bmask[j], B[i].y & gl.bmask[j]);
    }
  }
#pragma unroll
  for (int i = 0; i < NG; i++) {
    const float sx = __uint_as_float(Mt[i].y);
    const unsigned long long sc =
        fmul2(f2pack(h2f((uint16_t)(Ds[i] & 0xffffu)), h2f((uint16_t)(Ds[i] >> 16))), f2pack(sx, sx));
    const unsigned long long pm =
        f2pack(__int_as_float(D[i][0] * 256 + D[i][1]), __int_as_float(D[i][2] * 256 + D[i][3]));
    acc = ffma2(sc, fadd2(pm, f2pack(-kMagicF, -kMagicF)), acc);
  }
  a_adr += NG * 2 * kTileBytes;
  d_adr += NG * 2 * kTileBytes;
  b_adr += NG * 256;
  m_adr += NG * 32;
}

// the last tile of a slice with an odd tile count: blocks 0 / 1 of a group, two MMAs,
// lanes c = 0 / 1 extend their chains (lanes 2 / 3 have no block here)
__device__ __forceinline__ void gemv_half_group(uint32_t a_adr, uint32_t d_adr, uint32_t b_adr, uint32_t m_adr,
                                                const GemvLane& gl, int c, unsigned long long& acc) {
  const uint32_t m = 0x0f0f0f0fu;
  uint4 A;
  uint2 B, Mt = make_uint2(0u, 0u);
  uint32_t Ds = 0u;
  lds_u32x4(a_adr, A);
  lds_u32x2(b_adr, B);
  if (c < 2) {
    lds_u32x2(m_adr, Mt);
    asm("ld.shared.u32 %0, [%1];" : "=r"(Ds) : "r"(d_adr));
  }
  int D[4] = {0, (int)Mt.x, 0, (int)Mt.x};
  mma_u8s8_acc(D, A.x & m, A.y & m, (A.x >> 4) & m, (A.y >> 4) & m, B.x & gl.bmask[0], B.y & gl.bmask[0]);
  mma_u8s8_acc(D, A.z & m, A.w & m, (A.z >> 4) & m, (A.w >> 4) & m, B.x & gl.bmask[1], B.y & gl.bmask[1]);
  if (c < 2) {
    const float sx = __uint_as_float(Mt.y);
    const unsigned long long sc =
        fmul2(f2pack(h2f((uint16_t)(Ds & 0xffffu)), h2f((uint16_t)(Ds >> 16))), f2pack(sx, sx));
    const unsigned long long pm = f2pack(__int_as_float(D[0] * 256 + D[1]), __int_as_float(D[2] * 256 + D[3]));
    acc = ffma2(sc, fadd2(pm, f2pack(-kMagicF, -kMagicF)), acc);
  }
}

// per-stage GEMV constants (computed once per stage, not per task)
struct GemvDims {
  int kp, kp_blocks, tps;  // K parts, blocks per part, tiles per slice
  uint32_t xf, xm;         // staged x fragments / block meta (shared addresses)
  uint32_t xm2;            // Q6_K: half-block sums (shared address)
};

// One (unit, slice) task.  Returns the slice value of rows g / g + 8 in every lane of
// group g: ((chain 0 + chain 1) + (chain 2 + chain 3)).
__device__ __forceinline__ void gemv_task(const GemvDims& gd, uint32_t ubase, int kpi, int sl, int lane, float& acc0,
                                          float& acc1) {
  const int tps = gd.tps, g = lane >> 2, c = lane & 3;
  const int t0 = sl * tps;
  const int gb = kpi * gd.kp_blocks + 2 * t0;  // first block of the slice
  // per-lane addresses: A at lane * 16 of each tile; the scales of block c of the group
  // (rows g, g + 8) in tile c / 2 at 512 + 8 g + 4 (c % 2); digit entry lane of the group's
  // 4 blocks (256 B); the meta of block c
  uint32_t a_adr = ubase + (uint32_t)t0 * kTileBytes + lane * 16;
  uint32_t d_adr = ubase + (uint32_t)(t0 + (c >> 1)) * kTileBytes + 512 + g * 8 + (c & 1) * 4;
  uint32_t b_adr = gd.xf + (uint32_t)(gb * 8 + lane) * 8;
  uint32_t m_adr = gd.xm + (uint32_t)(gb + c) * 8;
  GemvLane gl;
#pragma unroll
  for (int j = 0; j < 4; j++) gl.bmask[j] = (lane >> 3) == j ? 0xffffffffu : 0u;
  unsigned long long acc = 0ull;  // (0.0f, 0.0f)
  int n = tps;
  for (; n >= 8; n -= 8) gemv_groups<4>(a_adr, d_adr, b_adr, m_adr, gl, acc);
  if (n >= 4) {
    gemv_groups<2>(a_adr, d_adr, b_adr, m_adr, gl, acc);
    n -= 4;
  }
  if (n >= 2) {
    gemv_groups<1>(a_adr, d_adr, b_adr, m_adr, gl, acc);
    n -= 2;
  }
  if (n) gemv_half_group(a_adr, d_adr, b_adr, m_adr, gl, c, acc);
  float e0, e1;
  f2unpack(acc, e0, e1);
  e0 = __fadd_rn(e0, __shfl_xor_sync(0xffffffffu, e0, 1));
  e1 = __fadd_rn(e1, __shfl_xor_sync(0xffffffffu, e1, 1));
  acc0 = __fadd_rn(e0, __shfl_xor_sync(0xffffffffu, e0, 2));
  acc1 = __fadd_rn(e1, __shfl_xor_sync(0xffffffffu, e1, 2));
}

// ------------------------------------------------------------------ batch GEMV
// One (unit, slice) task for NB sequences.  A 4-block group's integer MMAs multiply the
// NB sequences' digit columns together, the weight fragments loaded once:
//   NB <= 4: NB accumulator sets of CL = 4 / NB blocks; the MMA of block a CL + jc of set a
//            uses B columns 2 NB jc .. 2 NB jc + 2 NB - 1 = the h / l digits of the NB
//            sequences (one 256-B run of staged records, masked to the MMA as in the
//            one-sequence chain), so lane (g, c) ends with block a CL + c / NB of sequence
//            c % NB;
//   NB = 8:  two MMAs per block (sequences 0..3, 4..7), lane (g, c) ends with the block of
//            sequences c and c + 4.
// Either way a lane extends, per sequence, the chains c' = 0..3 of the one-sequence order
// (chain c' = blocks c', c' + 4, ... ascending, acc = fma(fp32(d) sx, P, acc)), and the
// slice value is ((chain 0 + chain 1) + (chain 2 + chain 3)) as there: each sequence's
// result is bit-identical to its one-sequence launch.  The MMA count per group is 4 for
// NB <= 4 and 8 for NB = 8 (the tensor instruction has the columns to spare).
template <int NB>
struct BatchShape {
  static constexpr int CL = NB >= 4 ? 1 : 4 / NB;   // blocks per accumulator set (NB <= 4)
  static constexpr int NA = NB == 8 ? 8 : NB;       // accumulator pairs per lane
  static constexpr int NV = NB == 8 ? 2 : 1;        // sequences per lane
};

// the group of NBLK (4, or 2 for the last tile of an odd tile count) blocks at the
// addresses, accumulated into acc; advances the addresses by one whole group
template <int NB, int NBLK>
__device__ __forceinline__ void gemv_group_b(uint32_t& a_adr, uint32_t& s_adr, uint32_t& b_adr, uint32_t& m_adr,
                                             int lane, unsigned long long (&acc)[BatchShape<NB>::NA]) {
  constexpr int CL = BatchShape<NB>::CL;
  constexpr int NSET = NB == 8 ? 2 * NBLK : (NBLK + CL - 1) / CL;
  const uint32_t m = 0x0f0f0f0fu;
  const int c = lane & 3;
  uint4 A[NBLK / 2];
  uint2 SC[NBLK / 2];
  uint2 B[NSET], Mt[NSET];
#pragma unroll
  for (int t = 0; t < NBLK / 2; t++) {
    lds_u32x4(a_adr + t * kTileBytes, A[t]);
    lds_u32x2(s_adr + t * kTileBytes, SC[t]);
  }
#pragma unroll
  for (int a = 0; a < NSET; a++) {
    lds_u32x2(b_adr + a * 256, B[a]);
    lds_u32x2(m_adr + a * 32, Mt[a]);
  }
  int D[NSET][4];
#pragma unroll
  for (int a = 0; a < NSET; a++) {
    D[a][0] = 0;
    D[a][1] = (int)Mt[a].x;
    D[a][2] = 0;
    D[a][3] = (int)Mt[a].x;
  }
#pragma unroll
  for (int a = 0; a < NSET; a++) {
#pragma unroll
    for (int jc = 0; jc < (NB == 8 ? 1 : CL); jc++) {
      const int j = NB == 8 ? a >> 1 : a * CL + jc;  // block of the group
      if (j < NBLK) {
        const uint4& w = A[j >> 1];
        const uint32_t w0 = (j & 1) ? w.z : w.x, w1 = (j & 1) ? w.w : w.y;
        const uint32_t bm = (NB >= 4 || (lane / (32 / CL)) == jc) ? 0xffffffffu : 0u;
        mma_u8s8_acc(D[a], w0 & m, w1 & m, (w0 >> 4) & m, (w1 >> 4) & m, B[a].x & bm, B[a].y & bm);
      }
    }
  }
#pragma unroll
  for (int a = 0; a < NSET; a++) {
    const int blk = NB == 8 ? a >> 1 : a * CL + c / NB;  // this lane's block in set a
    const uint2 sw = (NBLK == 4 && (blk >> 1)) ? SC[NBLK / 2 - 1] : SC[0];
    const uint32_t ds = (blk & 1) ? sw.y : sw.x;
    const float sx = __uint_as_float(Mt[a].y);
    const unsigned long long sc =
        fmul2(f2pack(h2f((uint16_t)(ds & 0xffffu)), h2f((uint16_t)(ds >> 16))), f2pack(sx, sx));
    const unsigned long long pm = f2pack(__int_as_float(D[a][0] * 256 + D[a][1]), __int_as_float(D[a][2] * 256 + D[a][3]));
    acc[a] = ffma2(sc, fadd2(pm, f2pack(-kMagicF, -kMagicF)), acc[a]);
  }
  a_adr += 2 * kTileBytes;
  s_adr += 2 * kTileBytes;
  b_adr += NB * 256;
  m_adr += NB * 32;
}

// lane (g, c): rows g / g + 8 of sequence c % NB (NB = 8: of sequences c and c + 4); for
// NB = 2 lanes c and c ^ 2 hold the same values
template <int NB>
__device__ __forceinline__ void gemv_task_b(const GemvDims& gd, uint32_t ubase, int kpi, int sl, int lane,
                                            float (&v0)[BatchShape<NB>::NV], float (&v1)[BatchShape<NB>::NV]) {
  constexpr int NA = BatchShape<NB>::NA;
  const int tps = gd.tps, g = lane >> 2, c = lane & 3;
  const int t0 = sl * tps;
  const int gb = kpi * gd.kp_blocks + 2 * t0;  // first block of the slice
  uint32_t a_adr = ubase + (uint32_t)t0 * kTileBytes + lane * 16;
  uint32_t s_adr = ubase + (uint32_t)t0 * kTileBytes + 512 + g * 8;
  uint32_t b_adr = gd.xf + (uint32_t)(gb * NB * 8 + lane) * 8;
  uint32_t m_adr = gd.xm + (uint32_t)(gb * NB + c) * 8;
  unsigned long long acc[NA];
#pragma unroll
  for (int a = 0; a < NA; a++) acc[a] = 0ull;
  int n = tps;
#pragma unroll(NB == 8 ? 1 : 2)
  for (; n >= 2; n -= 2) gemv_group_b<NB, 4>(a_adr, s_adr, b_adr, m_adr, lane, acc);
  if (n) gemv_group_b<NB, 2>(a_adr, s_adr, b_adr, m_adr, lane, acc);
  float e[NA][2];
#pragma unroll
  for (int a = 0; a < NA; a++) f2unpack(acc[a], e[a][0], e[a][1]);
  if constexpr (NB == 2) {  // set a: chains 2a + c / 2; partner c ^ 2 holds chain 2a + 1 - c / 2
#pragma unroll
    for (int a = 0; a < 2; a++)
#pragma unroll
      for (int r = 0; r < 2; r++) e[a][r] = __fadd_rn(e[a][r], __shfl_xor_sync(0xffffffffu, e[a][r], 2));
    v0[0] = __fadd_rn(e[0][0], e[1][0]);
    v1[0] = __fadd_rn(e[0][1], e[1][1]);
  } else if constexpr (NB == 4) {  // set a = chain a
    v0[0] = __fadd_rn(__fadd_rn(e[0][0], e[1][0]), __fadd_rn(e[2][0], e[3][0]));
    v1[0] = __fadd_rn(__fadd_rn(e[0][1], e[1][1]), __fadd_rn(e[2][1], e[3][1]));
  } else {  // set 2 j + h = chain j of sequence c + 4 h
#pragma unroll
    for (int h = 0; h < 2; h++) {
      v0[h] = __fadd_rn(__fadd_rn(e[h][0], e[2 + h][0]), __fadd_rn(e[4 + h][0], e[6 + h][0]));
      v1[h] = __fadd_rn(__fadd_rn(e[h][1], e[2 + h][1]), __fadd_rn(e[4 + h][1], e[6 + h][1]));
    }
  }
}

// ------------------------------------------------------------------ Q6_K (T6 units)
// Unit = 16 rows x Kp columns, 105 Kp / 8 bytes: the fp16 d of each 256-weight super-
// block for row pairs (g, g + 8) [Kp/256][8][2], the int8 scale of each 16-weight
// sub-block [Kp/16][8][2], then per 64 weights (two 32-weight tiles, one integer MMA
// each) 768 B: lane L's nibble words (16 B: per tile N0, N1) and high-bit words (8 B:
// per tile H).  For lane (g, c) of a tile, with A = q + 32 as u8:
//   N0 byte i = low(row g, k 4c + i) | low(row g, k 16 + 4c + i) << 4   (a0 | a2)
//   N1 byte i = the same for row g + 8                                    (a1 | a3)
//   H  byte i = high(a0_i) | high(a1_i) << 2 | high(a2_i) << 4 | high(a3_i) << 6
// (low = 4 bits, high = 2 bits).  B columns 0 / 1 carry the h / l digits of k 0..15
// (sub-block 0), columns 2 / 3 those of k 16..31 (sub-block 1); the accumulator input
// adds -32 sum X of the sub-block to its l column, so 256 D_h + D_l = sum q X.

// NT consecutive 32-weight tiles starting at tile t (all in one 256-weight super-block):
// all shared-memory loads, then the NT integer MMAs, then the scale / fma chain in tile
// order (the same order as one tile at a time)
template <int NT>
__device__ __forceinline__ void q6_tiles(uint32_t grp, uint32_t sc_pl, uint32_t d_pl, const GemvDims& gd, int kpi,
                                         int t, int lane, uint32_t m0, uint32_t m1, unsigned long long& acc) {
  const int g = lane >> 2, c = lane & 3;
  const uint32_t m = 0x0f0f0f0fu;
  uint2 nib[NT], B[NT], mt[NT], m2[NT];
  uint32_t H[NT];
  uint16_t scv[NT];
  if constexpr (NT % 2 == 0) {
    // t even: tiles (t + 2p, t + 2p + 1) share one 768-B group, whose 16 nibble bytes and
    // 8 high-bit bytes of this lane are one load each
#pragma unroll
    for (int p = 0; p < NT / 2; p++) {
      const uint32_t pb = grp + (uint32_t)((t >> 1) + p) * 768u;
      uint4 nn;
      uint2 hh;
      lds_u32x4(pb + lane * 16, nn);
      lds_u32x2(pb + 512 + lane * 8, hh);
      nib[2 * p] = make_uint2(nn.x, nn.y);
      nib[2 * p + 1] = make_uint2(nn.z, nn.w);
      H[2 * p] = hh.x;
      H[2 * p + 1] = hh.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < NT; j++) {
      const int tt = t + j;
      lds_u32x2(grp + (uint32_t)(tt >> 1) * 768u + lane * 16 + (tt & 1) * 8, nib[j]);
      asm("ld.shared.u32 %0, [%1];" : "=r"(H[j]) : "r"(grp + (uint32_t)(tt >> 1) * 768u + 512 + lane * 8 + (tt & 1) * 4));
    }
  }
#pragma unroll
  for (int j = 0; j < NT; j++) {
    const int tt = t + j, gb = kpi * gd.kp_blocks + tt;
    lds_u32x2(gd.xf + (uint32_t)(gb * 8 + (lane & 7)) * 8, B[j]);
    lds_u32x2(gd.xm + (uint32_t)gb * 8, mt[j]);
    lds_u32x2(gd.xm2 + (uint32_t)gb * 8, m2[j]);
    asm("ld.shared.u16 %0, [%1];" : "=h"(scv[j]) : "r"(sc_pl + (uint32_t)(2 * tt + (c & 1)) * 16 + g * 2));
  }
  uint32_t dv;
  asm("ld.shared.u32 %0, [%1];" : "=r"(dv) : "r"(d_pl + (uint32_t)(t >> 3) * 32 + g * 4));
  int D[NT][4];
#pragma unroll
  for (int j = 0; j < NT; j++) {
    const uint32_t a0 = (nib[j].x & m) | ((H[j] << 4) & 0x30303030u);
    const uint32_t a2 = ((nib[j].x >> 4) & m) | (H[j] & 0x30303030u);
    const uint32_t a1 = (nib[j].y & m) | ((H[j] << 2) & 0x30303030u);
    const uint32_t a3 = ((nib[j].y >> 4) & m) | ((H[j] >> 2) & 0x30303030u);
    const int corr = c == 0 ? (int)m2[j].x : (c == 1 ? (int)m2[j].y : 0);
    mma_u8s8(D[j], a0, a1, a2, a3, B[j].x & m0, B[j].y & m1, corr);
  }
  const unsigned long long dpair = f2pack(h2f((uint16_t)(dv & 0xffffu)), h2f((uint16_t)(dv >> 16)));
#pragma unroll
  for (int j = 0; j < NT; j++) {
    const float sx = __uint_as_float(mt[j].y);
    const unsigned long long scp =
        fmul2(fmul2(dpair, f2pack((float)(int8_t)(scv[j] & 0xff), (float)(int8_t)(scv[j] >> 8))), f2pack(sx, sx));
    acc = ffma2(scp, f2pack((float)(D[j][0] * 256 + D[j][1]), (float)(D[j][2] * 256 + D[j][3])), acc);
  }
}

// one Q6_K slice: lanes 4g (c = 0) return rows g / g + 8: the even sub-blocks' chain
// (c = 0) plus the odd sub-blocks' chain (c = 1)
__device__ __forceinline__ void gemv_task_q6(const GemvDims& gd, uint32_t ubase, int kpi, int t0, int ntiles, int lane,
                                             float& acc0, float& acc1) {
  const int n = lane >> 2;
  const int kp_cols = gd.kp_blocks * 32;
  const uint32_t d_pl = ubase, sc_pl = ubase + kp_cols / 8, grp = ubase + kp_cols / 8 + kp_cols;
  // B: the T16 staging's digit entry of this lane, masked to the lane's column block
  const uint32_t m0 = n < 2 ? 0xffffffffu : 0u, m1 = (n == 2 || n == 3) ? 0xffffffffu : 0u;
  unsigned long long acc = 0ull;
  int t = t0;
  const int te = t0 + ntiles;
  for (; t < te && (t & 3); t++) q6_tiles<1>(grp, sc_pl, d_pl, gd, kpi, t, lane, m0, m1, acc);
  for (; t + 4 <= te; t += 4) q6_tiles<4>(grp, sc_pl, d_pl, gd, kpi, t, lane, m0, m1, acc);
  for (; t < te; t++) q6_tiles<1>(grp, sc_pl, d_pl, gd, kpi, t, lane, m0, m1, acc);
  float e0, e1;
  f2unpack(acc, e0, e1);
  // chain of the odd sub-blocks (lane c = 1) onto the even one (lane c = 0)
  acc0 = __fadd_rn(e0, __shfl_xor_sync(0xffffffffu, e0, 1));
  acc1 = __fadd_rn(e1, __shfl_xor_sync(0xffffffffu, e1, 1));
}

__device__ __forceinline__ uint16_t bf16r(float v) { return f2bf(v); }

// epilogue of one row pair (positions g and g + 8 of unit u); Spark: the qkv stage's
// partial RoPE and gate rows, the GELU * mul epilogue.  NB > 1: of sequence bq (outputs
// at bq times their one-sequence size; rope_cs is that sequence's row, kvo its cache
// offset)
template <bool Spark, int NB = 1>
__device__ __forceinline__ void gemv_epilogue(const SparkStage& st, const SparkStepIO& io, const long long* misc64,
                                              const uint16_t* rope_cs, int u, int g, float v0, float v1,
                                              unsigned long long& best, int bq = 0, long long kvo = 0) {
  const int rg = u / st.kp, kpi = u - rg * st.kp;
  int r0, r1;
  if constexpr (Spark) {
    const int aux = st.head_dim | (st.rotary_dim << 16);
    r0 = t16_row_x(st.rowmap, rg, g, st.n, aux);
    r1 = t16_row_x(st.rowmap, rg, g + 8, st.n, aux);
  } else {
    r0 = t16_row(st.rowmap, rg, g, st.n, st.head_dim);
    r1 = t16_row(st.rowmap, rg, g + 8, st.n, st.head_dim);
  }
  switch (st.epi) {
    case SPARK_EPI_BF16: {
      uint16_t* y = static_cast<uint16_t*>(st.out) + (NB > 1 ? (size_t)bq * st.n : 0);
      y[r0] = bf16r(v0);
      y[r1] = bf16r(v1);
      break;
    }
    case SPARK_EPI_PARTS: {
      if (st.xchg == SPARK_XCHG_TAGGED) {  // tagged words (value | tag << 32), into every rank's window
        const unsigned long long tag = (unsigned long long)(uint32_t)(misc64[2] + 1) << 32;
        unsigned long long* y = static_cast<unsigned long long*>(st.out) + (size_t)(io.tp_rank * st.kp + kpi) * st.n;
        for (int p = 0; p < io.tp_size; p++) {
          unsigned long long* yp = peer_addr(io, p, y);
          asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(yp + r0), "l"(tag | __float_as_uint(v0))
                       : "memory");
          asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(yp + r1), "l"(tag | __float_as_uint(v1))
                       : "memory");
        }
      } else if (st.xchg) {  // part tp_rank * kp + kpi, into every rank's window
        float* y = static_cast<float*>(st.out) + (size_t)(io.tp_rank * st.kp + kpi) * st.n;
        for (int p = 0; p < io.tp_size; p++) {
          float* yp = peer_addr(io, p, y);
          yp[r0] = v0;
          yp[r1] = v1;
        }
      } else {
        float* y = static_cast<float*>(st.out) + (size_t)((NB > 1 ? bq * st.kp : 0) + kpi) * st.n;
        y[r0] = v0;
        y[r1] = v1;
      }
      break;
    }
    case SPARK_EPI_SILU_MUL: {
      const float gf = bf2f(f2bf(v0)), uf = bf2f(f2bf(v1));
      const float act = bf2f(f2bf(__fdiv_rn(gf, __fadd_rn(1.0f, spark_exp(-gf)))));
      static_cast<uint16_t*>(st.out)[(NB > 1 ? (size_t)bq * (st.n >> 1) : 0) + r0] = f2bf(__fmul_rn(act, uf));
      break;
    }
    case SPARK_EPI_GELU_MUL: {
      if constexpr (Spark) {
        const float act = bf2f(spark_gelu_bf16(f2bf(v0), static_cast<const uint16_t*>(st.table)));
        static_cast<uint16_t*>(st.out)[r0] = f2bf(__fmul_rn(act, bf2f(f2bf(v1))));
      }
      break;
    }
    case SPARK_EPI_ARGMAX: {
      const uint16_t b0 = f2bf(v0), b1 = f2bf(v1);
      if (st.out) {
        uint16_t* y = static_cast<uint16_t*>(st.out) + (NB > 1 ? (size_t)bq * st.n : 0);
        y[r0] = b0;
        y[r1] = b1;
      }
      const unsigned long long k0 = argmax_key(b0, st.row0 + r0), k1 = argmax_key(b1, st.row0 + r1);
      const unsigned long long k = k0 > k1 ? k0 : k1;
      best = k > best ? k : best;
      break;
    }
    default: {  // SPARK_EPI_ROPE_KV
      const int D = st.head_dim;
      int half = D >> 1;
      const int hd = r0 / D, i = r0 - hd * D;
      float a = bf2f(f2bf(v0)), b = bf2f(f2bf(v1));
      bool rot = hd < st.nq + st.nkv;
      if constexpr (Spark) {
        const int nh = st.nq + 2 * st.nkv;
        if (hd >= nh) {  // gate rows: g = bf16(sigmoid(bf16(logit))) of head r - nh D
          const int h0 = r0 - nh * D, h1 = r1 - nh * D;
          uint16_t* gt = static_cast<uint16_t*>(st.gate);
          if (h0 < st.nq) gt[h0] = f2bf(__fdiv_rn(1.0f, __fadd_rn(1.0f, spark_exp(-a))));
          if (h1 < st.nq) gt[h1] = f2bf(__fdiv_rn(1.0f, __fadd_rn(1.0f, spark_exp(-b))));
          break;
        }
        const int r = st.rotary_dim ? st.rotary_dim : D;
        if (i < (r >> 1)) {
          half = r >> 1;
        } else {  // the head's dims past the rotary part: plain rows i and i + 8
          half = 8;
          rot = false;
        }
      }
      if (rot) {
        const float c = bf2f(rope_cs[i]), sn = bf2f(rope_cs[i + half]);
        const float u2 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
        const float w2 = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, sn));
        a = u2;
        b = w2;
      }
      const uint16_t ua = f2bf(a), ub = f2bf(b);
      if (hd < st.nq) {
        uint16_t* q = static_cast<uint16_t*>(st.q) + ((NB > 1 ? (size_t)bq * st.nq : 0) + hd) * D;
        q[i] = ua;
        q[i + half] = ub;
      } else {
        const int isv = hd >= st.nq + st.nkv;
        const int hk = hd - st.nq - isv * st.nkv;
        uint16_t* cache = static_cast<uint16_t*>(isv ? st.v_cache : st.k_cache);
        uint16_t* dst = cache + (NB > 1 ? kvo : misc64[1]) + (int64_t)hk * st.block_size * D;
        dst[i] = ua;
        dst[i + half] = ub;
        uint16_t* kn =
            static_cast<uint16_t*>(st.kv_new) + ((NB > 1 ? (size_t)bq * 2 * st.nkv : 0) + (size_t)isv * st.nkv + hk) * D;
        kn[i] = ua;
        kn[i + half] = ub;
      }
      break;
    }
  }
}

// Wait until ring sequence `seq` has landed.  A parity wait alone cannot tell a slot two
// phases behind (its previous copy, seq - kDesc, still in flight) from a completed one, and
// warps move through the ring out of step with each other (attention ranges, GEMV tasks),
// so the wait first sees the slot's issue tag equal `seq`: the producer issues seq only
// after seq - kDesc was released, hence landed, and cannot issue seq + kDesc before this
// warp releases seq.  Both waits are bounded like every other.
__device__ __forceinline__ bool wait_unit(const Smem& s, uint32_t seq) {
  const volatile uint32_t* tag = s.desc_seq + seq % kDesc;
  if (*tag != seq) {
    unsigned long long t0 = 0;
    for (uint32_t i = 0; *tag != seq; i++) {
      if ((i & 255) == 255) {
        if (*s.abort_flag) return false;
        const unsigned long long t = gtimer();
        if (t0 == 0) t0 = t;
        else if (t - t0 > kWaitNs) return false;
      }
    }
  }
  return mbar_wait_timed(smem_u32(s.full + seq % kDesc), (seq / kDesc) & 1u, s.abort_flag);
}


// Q6: the kernel instantiation that also runs SPARK_STAGE_GEMV_Q6 stages (programs
// without them use the Q4-only instantiation, whose registers the Q6 code does not touch)
template <bool Q6, bool Spark, bool TP>
__device__ __forceinline__ bool gemv_stage(const StepParams& P, const SparkStage& st, const Smem& s, uint32_t& seq_base, int tid) {
  const int ncta = gridDim.x, cta = blockIdx.x, warp = tid >> 5, lane = tid & 31;
  int u0, ustride;
  const int nl = local_units(st, cta, ncta, u0, ustride);
  // the CTA's K part alone is staged when all its units share it (SPARK_PRO_ATTN: staged
  // already, by the attention stage before)
  const bool pro_attn = st.pro == SPARK_PRO_ATTN;
  const bool part_x = pro_attn || (!st.norm && st.kp > 1 && ncta % st.kp == 0);
  const int kx = part_x ? st.k / st.kp : st.k;
  if (!pro_attn && (nl > 0 || (cta == 0 && st.res_out)))
    stage_x<Q6, TP>(P, st, s, tid,
            (tid == 0 && P.io.trace) ? P.io.trace + ((size_t)cta * P.num_stages + s.flag[2]) * kTraceSlots : nullptr,
            part_x ? (u0 % st.kp) * kx : 0, kx);
  consumer_bar();
  unsigned long long* tr = (tid == 0 && P.io.trace)
                               ? P.io.trace + ((size_t)cta * P.num_stages + s.flag[2]) * kTraceSlots
                               : nullptr;
  if (tr) tr[4] = gtimer();
  unsigned long long best = 0ull;
  const int ks = st.ks;
  GemvDims gd;
  gd.kp = st.kp;
  gd.kp_blocks = (st.k / st.kp) >> 5;
  gd.tps = (gd.kp_blocks >> 1) / ks;
  gd.xf = smem_u32(s.scratch);
  gd.xm = gd.xf + 64 * (kx >> 5);
  gd.xm2 = gd.xf + 72 * (kx >> 5) + 6 * st.k;  // Q6_K half-block sums (stage_x)
  unsigned long long wsum = 0;  // trace: warp 0's time waiting for ring data (ns)
  long long csum = 0;           // trace: warp 0's SM cycles inside its GEMV tasks
  long long psum = 0;           // trace: ... after them (slice sums, epilogue, slot release)
  const long long cloop = tr ? clock64() : 0ll;
  int ntask = 0;
  for (int t = warp; t < nl * ks; t += kWarps) {
    const int j = t / ks, sl = t - j * ks;
    const uint32_t seq = seq_base + j;
    const unsigned long long w0 = tr ? gtimer() : 0ull;
    if (!wait_unit(s, seq)) {  // abort: skip the work, keep the barriers
      raise_abort(P, s, SPARK_ERR_LAUNCH);
      continue;
    }
    if (tr) {
      wsum += gtimer() - w0;
      ntask++;
    }
    const long long c0 = tr ? clock64() : 0ll;
    const int u = u0 + j * ustride;
    const uint32_t slot = seq % kDesc;
    float acc0, acc1;
    if (Q6 && st.kind == SPARK_STAGE_GEMV_Q6) {
      const int tq = gd.kp_blocks / ks;  // 32-weight tiles per slice
      gemv_task_q6(gd, smem_u32(s.ring) + s.desc_off[slot], part_x ? 0 : u % gd.kp, sl * tq, tq, lane, acc0, acc1);
    } else {
      gemv_task(gd, smem_u32(s.ring) + s.desc_off[slot], part_x ? 0 : u % gd.kp, sl, lane, acc0, acc1);
    }
    const long long c1 = tr ? clock64() : 0ll;
    if (tr) csum += c1 - c0;
    if (ks == 1) {  // the unit is this task: lane g takes rows g / g + 8 from lane 4 g
      const float v0 = __shfl_sync(0xffffffffu, acc0, 4 * (lane & 7));
      const float v1 = __shfl_sync(0xffffffffu, acc1, 4 * (lane & 7));
      if (lane < 8) gemv_epilogue<Spark>(st, P.io, s.misc64, s.rope_cs, u, lane, v0, v1, best);
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(s.empty + slot));
    } else {
      float* pr = s.partial + slot * kMaxSlices * 16;
      if ((lane & 3) == 0) {
        pr[sl * 16 + (lane >> 2)] = acc0;
        pr[sl * 16 + (lane >> 2) + 8] = acc1;
      }
      // the task that completes the unit sums its slices, runs the epilogue and frees the
      // slot: the warp's slice sums (ordered by the warp barrier) are released, and the
      // other slices' acquired, by lane 0's acquire-release count
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        int old;
        asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;" : "=r"(old) : "r"(smem_u32(s.done + slot))
                     : "memory");
        last = old == ks - 1;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      __syncwarp();
      if (last) {
        if (lane < 8) {
          float v0 = pr[lane], v1 = pr[lane + 8];
          for (int q = 1; q < ks; q++) {
            v0 = __fadd_rn(v0, pr[q * 16 + lane]);
            v1 = __fadd_rn(v1, pr[q * 16 + lane + 8]);
          }
          gemv_epilogue<Spark>(st, P.io, s.misc64, s.rope_cs, u, lane, v0, v1, best);
        }
        __syncwarp();
        if (lane == 0) {
          s.done[slot] = 0;
          mbar_arrive(smem_u32(s.empty + slot));
        }
      }
    }
    if (tr) psum += clock64() - c1;
  }
  if (tr) {
    tr[5] = gtimer();
    tr[12] = (unsigned long long)psum;
    tr[13] = (unsigned long long)(clock64() - cloop);
    tr[8] = (unsigned long long)csum;
    tr[9] = wsum;
    tr[11] = (unsigned long long)ntask * (unsigned long long)(Q6 && st.kind == SPARK_STAGE_GEMV_Q6 ? gd.kp_blocks / ks
                                                                                                  : gd.tps);
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
      if (m) {
        if (st.xchg) {
          for (int p = 0; p < P.io.tp_size; p++) atomicMax_system(peer_addr(P.io, p, st.key), m);
        } else {
          atomicMax(st.key, m);
        }
      }
    }
  }
  seq_base += nl;
  return true;
}


// A GEMV stage of a batch-NB program: the one-sequence stage's units, tasks and slot
// handling, with NB staged inputs, the batch task and NB epilogues per row pair (lane
// (g, c) runs those of its sequences c % NB, c < NB; NB = 8: c and c + 4).  Slice sums:
// [slot][slice][sequence][16].
template <int NB>
__device__ __forceinline__ bool gemv_stage_b(const StepParams& P, const SparkStage& st, const Smem& s, uint32_t& seq_base,
                                             int tid) {
  constexpr int NV = BatchShape<NB>::NV;
  const int ncta = gridDim.x, cta = blockIdx.x, warp = tid >> 5, lane = tid & 31, c = lane & 3;
  int u0, ustride;
  const int nl = local_units(st, cta, ncta, u0, ustride);
  const bool part_x = !st.norm && st.kp > 1 && ncta % st.kp == 0;
  const int kx = part_x ? st.k / st.kp : st.k;
  unsigned long long* tr = (tid == 0 && P.io.trace)
                               ? P.io.trace + ((size_t)cta * P.num_stages + s.flag[2]) * kTraceSlots
                               : nullptr;
  if (nl > 0 || (cta == 0 && st.res_out)) stage_x_batch<NB>(st, s, tid, tr, part_x ? (u0 % st.kp) * kx : 0, kx);
  consumer_bar();
  if (tr) tr[4] = gtimer();
  const bool owner = NB >= 4 || c < NB;
  int bqs[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) bqs[i] = NB == 8 ? c + 4 * i : c % NB;
  unsigned long long best[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) best[i] = 0ull;
  const int ks = st.ks;
  GemvDims gd;
  gd.kp = st.kp;
  gd.kp_blocks = (st.k / st.kp) >> 5;
  gd.tps = (gd.kp_blocks >> 1) / ks;
  gd.xf = smem_u32(s.scratch);
  gd.xm = gd.xf + 64 * (kx >> 5) * NB;
  gd.xm2 = 0;
  const bool rope = st.epi == SPARK_EPI_ROPE_KV;
  auto epi = [&](int u, int g, int i, float v0, float v1) {
    const int bq = bqs[i];
    gemv_epilogue<false, NB>(st, P.io, s.misc64, rope ? s.rope_cs + 128 * bq : s.rope_cs, u, g, v0, v1, best[i], bq,
                             rope ? s.bkvoff[bq] : 0ll);
  };
  for (int t = warp; t < nl * ks; t += kWarps) {
    const int j = t / ks, sl = t - j * ks;
    const uint32_t seq = seq_base + j;
    if (!wait_unit(s, seq)) {  // abort: skip the work, keep the barriers
      raise_abort(P, s, SPARK_ERR_LAUNCH);
      continue;
    }
    const int u = u0 + j * ustride;
    const uint32_t slot = seq % kDesc;
    float v0[NV], v1[NV];
    gemv_task_b<NB>(gd, smem_u32(s.ring) + s.desc_off[slot], part_x ? 0 : u % gd.kp, sl, lane, v0, v1);
    if (ks == 1) {
      if (owner)
#pragma unroll
        for (int i = 0; i < NV; i++) epi(u, lane >> 2, i, v0[i], v1[i]);
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(s.empty + slot));
    } else {
      float* pr = s.partial + slot * Layout<NB>::slices * 16 * NB;
      if (owner) {
#pragma unroll
        for (int i = 0; i < NV; i++) {
          pr[(sl * NB + bqs[i]) * 16 + (lane >> 2)] = v0[i];
          pr[(sl * NB + bqs[i]) * 16 + (lane >> 2) + 8] = v1[i];
        }
      }
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        int old;
        asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;" : "=r"(old) : "r"(smem_u32(s.done + slot))
                     : "memory");
        last = old == ks - 1;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      __syncwarp();
      if (last) {
        if (owner) {
#pragma unroll
          for (int i = 0; i < NV; i++) {
            const int g = lane >> 2, bq = bqs[i];
            float a0 = pr[bq * 16 + g], a1 = pr[bq * 16 + g + 8];
            for (int q = 1; q < ks; q++) {
              a0 = __fadd_rn(a0, pr[(q * NB + bq) * 16 + g]);
              a1 = __fadd_rn(a1, pr[(q * NB + bq) * 16 + g + 8]);
            }
            epi(u, g, i, a0, a1);
          }
        }
        __syncwarp();
        if (lane == 0) {
          s.done[slot] = 0;
          mbar_arrive(smem_u32(s.empty + slot));
        }
      }
    }
  }
  if (tr) tr[5] = gtimer();
  if (st.epi == SPARK_EPI_ARGMAX) {  // per sequence: over the lanes of the same c, the warps, the CTAs
#pragma unroll
    for (int i = 0; i < NV; i++) {
#pragma unroll
      for (int off = 16; off >= 4; off /= 2) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, best[i], off);
        best[i] = o > best[i] ? o : best[i];
      }
      if (lane < 4 && owner) s.red64[warp * NB + bqs[i]] = best[i];
    }
    consumer_bar();
    if (tid < NB) {
      unsigned long long m = 0;
      for (int w = 0; w < kWarps; w++) m = s.red64[w * NB + tid] > m ? s.red64[w * NB + tid] : m;
      if (m) atomicMax(st.key + tid, m);
    }
  }
  seq_base += nl;
  return true;
}

// ------------------------------------------------------------------ consumers: attention
// Task (kv head g, split j): tokens [t0, t1) of the context pos + 1 (Spark sliding
// window: of its last `window` positions), T = split_len.  Head dim D = 128 (256 in the
// Spark instantiation).  The split's n tokens are cut into kWarps contiguous ranges of
// C = roundup(ceil(n / kWarps), TPI) tokens (TPI = 512 / D tokens per warp step); warp w
// runs a softmax of its own over range w: scores with D / 16 lanes per token (lane jj owns
// dims 8jj..8jj+7 and D/2+8jj..; even / odd positions in two fma chains, xor butterfly
// over the token's lanes), m_w = the range's maximum, p = exp(s - m_w) with lane i mod 32
// of the range summing l_w (butterfly), P = bf16(p), O_w = sum over the range of P V
// (lane owns D / 32 dims of the 4 heads, tokens ascending).  The CTA merges the ranges in
// warp order: M = max m_w, f_w = exp(m_w - M), L = L + f_w l_w, O = O + f_w O_w; the
// split's partial is O / L with lse = log(L) + M.  No CTA barrier separates a warp's
// scores, softmax and P V.
//
// The combine of a kv head's S partials (the oracle's combine order: M = max lse,
// w_s = exp(lse_s - M) / sum, out = bf16(sum w_s O_s); Spark: times the head's gate) is
// done by every CTA of the head when the next stage is a SPARK_PRO_ATTN o_proj (its
// input then stays in shared memory), else by the split that completes the head last
// (no CTA waits for another).
// combine: a head group's partials pass through the scratch in rounds of whole splits
constexpr int kCombineBytes = 36 * 1024;          // partials of one round
constexpr int kCombineLseOff = kCombineBytes;     // lse [4][S], weights [4][S], maxima [4]
constexpr int kMaxCombineSplits = (kScratchBytes - kCombineLseOff - 16) / 32;
constexpr int kXinOff = 32 * 1024;                // combined output (bf16) before the o_proj staging

// the decoded token's K and V rows (2 x D bf16), copied from kv_new by the range that
// holds it, past the split's scores and P
constexpr int kKvNewOff = 24 * kMaxSplitTokens;
static_assert(kKvNewOff % 16 == 0 && kKvNewOff + 4 * 256 <= kScratchBytes, "kv_new rows in the scratch");

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__host__ __device__ __forceinline__ int warp_range(int n, int tpi) {
  const int c = (n + kWarps - 1) / kWarps;
  return (c + tpi - 1) / tpi * tpi;
}

// Ring runs seq0 + r0 .. seq0 + r1 (K or V runs of the split [t0, t1) starting at run w0)
// are done for this warp: lane 0 counts each, and the last of the warps whose range
// touches a run (range w = [w C, w C + C) of the split) frees its ring bytes.  A run is
// only freed after it has landed (the run of the decoded token alone is never read from
// the ring, so the range may not have waited on it).
__device__ __forceinline__ void release_runs(const Smem& s, uint32_t seq0, int r0, int r1, int64_t t0, int64_t t1,
                                             int64_t w0, int C, int lane) {
  if (lane == 0) {
    for (int r = r0; r <= r1; r++) {
      if (!wait_unit(s, seq0 + r)) break;  // (abort: the producer no longer issues)
      const int64_t rs = ((w0 + r) * kRunTokens > t0 ? (w0 + r) * kRunTokens : t0) - t0;
      const int64_t re = ((w0 + r + 1) * kRunTokens < t1 ? (w0 + r + 1) * kRunTokens : t1) - t0;
      const int nw = (int)((re - 1) / C - rs / C + 1);
      const uint32_t slot = (seq0 + r) % kDesc;
      if (atomicAdd(s.done + slot, 1) == nw - 1) {
        s.done[slot] = 0;
        mbar_arrive(smem_u32(s.empty + slot));
      }
    }
  }
  __syncwarp();
}

// One task (kv head g, split j): the ranges' softmax and P V, their merge, the split's
// partials.  false: the split is longer than the scratch holds (launch aborted).  NB > 1:
// of sequence bq (its position, q, kv_new and partials).
template <int D, bool Spark, int NB = 1>
__device__ __forceinline__ bool attn_split(const StepParams& P, const SparkStage& st, const Smem& s, uint32_t& seq_base,
                                           int tid, int g, int j, int bq = 0) {
  const int warp = tid >> 5, lane = tid & 31;
  const int nq = st.nq, S = st.splits;
  const int64_t pos = NB > 1 ? s.bpos[bq] : s.misc64[0], len = pos + 1;
  // Spark sliding window: positions [lo, len); the splits start at lo rounded down to 16,
  // positions before lo score -inf
  const int64_t lo = Spark && st.window > 0 && len > st.window ? len - st.window : 0;
  const int64_t start = lo & ~(int64_t)15;
  const int T = split_len(len - start, S);
  if (T > kMaxSplitTokens) {
    if (tid == 0) raise_abort(P, s, SPARK_ERR_TOO_LARGE);
    return false;
  }
  const int64_t t0 = start + (int64_t)j * T, t1 = t0 + T < len ? t0 + T : len;
  const int n = t1 > t0 ? (int)(t1 - t0) : 0;
  float* part_o = st.part_o + (NB > 1 ? (size_t)bq * S * nq * D : 0);
  float* part_lse = st.part_lse + (NB > 1 ? (size_t)bq * S * nq : 0);
  const uint16_t* kv_new = static_cast<const uint16_t*>(st.kv_new) + (NB > 1 ? (size_t)bq * 2 * st.nkv * D : 0);
  unsigned long long* tr = (tid == 0 && P.io.trace)
                               ? P.io.trace + ((size_t)blockIdx.x * P.num_stages + s.flag[2]) * kTraceSlots
                               : nullptr;
  const float ninf = __int_as_float(0xff800000);
  if (n == 0) {
    for (int o = tid; o < 4 * D; o += kConsumers) part_o[((size_t)j * nq + 4 * g) * D + o] = 0.0f;
    if (tid < 4) part_lse[(size_t)j * nq + 4 * g + tid] = ninf;
    return true;
  }
  const int64_t w0 = t0 / kRunTokens;
  const int nruns = (int)((t1 - 1) / kRunTokens - w0 + 1);
  constexpr int LPT = D / 16, TPI = 32 / LPT, DL = D / 32;
  const int jj = lane & (LPT - 1), grp = lane / LPT;
  const int C = warp_range(n, TPI);
  const int a = warp * C, b = a + C < n ? a + C : n;  // this warp's range (empty when a >= n)
  float4* rec = reinterpret_cast<float4*>(s.scratch);             // [T] scores of the 4 heads
  uint2* pbf = reinterpret_cast<uint2*>(s.scratch + 16 * T);      // [T] bf16 P of the 4 heads
  float mx[4] = {ninf, ninf, ninf, ninf}, l[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  float acc[4][DL];
#pragma unroll
  for (int h = 0; h < 4; h++)
#pragma unroll
    for (int d = 0; d < DL; d++) acc[h][d] = 0.0f;
  bool ok = true;
  cstamp(tr, 12);
  // The token being decoded (pos, the last token of the last split) is peeled off both
  // loops: its K / V come from kv_new (this launch's qkv stage wrote them; the ring's copy
  // of its run predates that), so the loops themselves read shared memory only.  Its two
  // rows are copied into the scratch together with the q loads, so their L2 round trip
  // overlaps the scores instead of following them.
  const bool has_pos = a < b && pos >= t0 + a && pos < t0 + b;  // then pos = t0 + b - 1
  if (has_pos) {
    const uint32_t kvs = smem_u32(s.scratch + kKvNewOff);
    const uint16_t* kr = kv_new + (size_t)g * D;
    const uint16_t* vr = kv_new + ((size_t)st.nkv + g) * D;
    for (int c = lane; c < 2 * (D / 8); c += 32) cp_async16(kvs + 16 * c, c < D / 8 ? kr + 8 * c : vr + 8 * (c - D / 8));
  }
  if (a < b) {
    float qf[4][16];
    {
      const uint16_t* q = static_cast<const uint16_t*>(st.q) + ((NB > 1 ? (size_t)bq * nq : 0) + (size_t)4 * g) * D;
#pragma unroll
      for (int h = 0; h < 4; h++) {
        float lo8[8], hi8[8];
        unpack8(__ldcg(reinterpret_cast<const uint4*>(q + h * D + 8 * jj)), lo8);
        unpack8(__ldcg(reinterpret_cast<const uint4*>(q + h * D + D / 2 + 8 * jj)), hi8);
#pragma unroll
        for (int m = 0; m < 8; m++) {
          qf[h][m] = lo8[m];
          qf[h][8 + m] = hi8[m];
        }
      }
    }
    if (tr) {  // trace: the q loads have returned (the clock read takes the last q value as input)
      unsigned long long t;
      asm volatile("mov.u64 %0, %%clock64;" : "=l"(t) : "f"(qf[3][15]));
      tr[23] = t;
    }
    const int bl = has_pos ? b - 1 : b;                  // ring tokens of the range: [a, bl)
    // ---- scores (a TPI-token step never crosses a 64-token run: t0 and a are multiples of TPI)
    int waited = -1;
    const unsigned char* rowbase = nullptr;
    int64_t rs = 0;
    auto dot4 = [&](const uint4& k0, const uint4& k1, float (&sc)[4]) {
      const uint32_t kw[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
      for (int h = 0; h < 4; h++) {
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
        for (int m = 0; m < 8; m++) {
          a0 = __fmaf_rn(qf[h][2 * m], bf_lo(kw[m]), a0);
          a1 = __fmaf_rn(qf[h][2 * m + 1], bf_hi(kw[m]), a1);
        }
        float v = __fadd_rn(a0, a1);
        if constexpr (LPT == 16) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 8));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
        sc[h] = __fmul_rn(v, st.scale);
      }
    };
    for (int i0 = a; i0 < bl; i0 += TPI) {
      const int r = (int)((t0 + i0) / kRunTokens - w0);
      if (r != waited) {
        if (!wait_unit(s, seq_base + r)) {
          ok = false;
          break;
        }
        waited = r;
        rs = (w0 + r) * kRunTokens > t0 ? (w0 + r) * kRunTokens : t0;
        rowbase = s.ring + s.desc_off[(seq_base + r) % kDesc];
      }
      const int i = i0 + grp;
      const bool in = i < bl;
      const bool valid = in && (!Spark || t0 + i >= lo);
      uint4 k0 = make_uint4(0, 0, 0, 0), k1 = k0;
      if (in) {
        const unsigned char* kr = rowbase + (t0 + i - rs) * (2 * D);
        k0 = *reinterpret_cast<const uint4*>(kr + 16 * jj);
        k1 = *reinterpret_cast<const uint4*>(kr + D + 16 * jj);
      }
      float sc[4];
      dot4(k0, k1, sc);
#pragma unroll
      for (int h = 0; h < 4; h++)
        if (valid) mx[h] = sc[h] > mx[h] ? sc[h] : mx[h];
      if (jj == 0 && in) rec[i] = valid ? make_float4(sc[0], sc[1], sc[2], sc[3]) : make_float4(ninf, ninf, ninf, ninf);
    }
    if (has_pos) {  // the warp's copies of the decoded token's rows
      cp_async_wait_all();
      __syncwarp();
    }
    if (ok && has_pos) {  // every lane group scores the decoded token; group 0 stores it
      const unsigned char* kvn = s.scratch + kKvNewOff;
      const uint4 k0 = *reinterpret_cast<const uint4*>(kvn + 16 * jj);
      const uint4 k1 = *reinterpret_cast<const uint4*>(kvn + D + 16 * jj);
      float sc[4];
      dot4(k0, k1, sc);
#pragma unroll
      for (int h = 0; h < 4; h++) mx[h] = sc[h] > mx[h] ? sc[h] : mx[h];
      if (lane == 0) rec[b - 1] = make_float4(sc[0], sc[1], sc[2], sc[3]);
    }
    cstamp(tr, 13);
    const int r0 = (int)((t0 + a) / kRunTokens - w0), r1 = (int)((t0 + b - 1) / kRunTokens - w0);
    if (ok) release_runs(s, seq_base, r0, r1, t0, t1, w0, C, lane);  // K runs
    if (ok) {
      // ---- the range's maximum, p = exp(s - m_w), l_w (lane i mod 32 of the range), P = bf16(p)
#pragma unroll
      for (int h = 0; h < 4; h++)
#pragma unroll
        for (int off = LPT; off < 32; off <<= 1) {
          const float o = __shfl_xor_sync(0xffffffffu, mx[h], off);
          mx[h] = o > mx[h] ? o : mx[h];
        }
      __syncwarp();
      for (int i = a + lane; i < b; i += 32) {
        const float4 s4 = rec[i];
        const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
        float pv[4];
#pragma unroll
        for (int h = 0; h < 4; h++) {
          pv[h] = mx[h] == ninf ? 0.0f : spark_exp_neg(__fsub_rn(sv[h], mx[h]));
          l[h] = __fadd_rn(l[h], pv[h]);
        }
        pbf[i] = make_uint2(bf16x2(pv[0], pv[1]), bf16x2(pv[2], pv[3]));
      }
#pragma unroll
      for (int h = 0; h < 4; h++) l[h] = butterfly_sum<32>(l[h]);
      __syncwarp();
      cstamp(tr, 14);
      // ---- P V over the range, tokens ascending: run by run, four tokens per batch (all
      // shared-memory loads first), then the decoded token from kv_new
      const uint32_t pbf_u = smem_u32(pbf);
      auto pv_token = [&](uint2 pw, const float (&v4)[DL]) {
        const float p4[4] = {bf_lo(pw.x), bf_hi(pw.x), bf_lo(pw.y), bf_hi(pw.y)};
#pragma unroll
        for (int h = 0; h < 4; h++)
#pragma unroll
          for (int d = 0; d < DL; d++) acc[h][d] = __fmaf_rn(p4[h], v4[d], acc[h][d]);
      };
      auto v_load = [&](uint32_t adr, float (&v4)[DL]) {
        if constexpr (D == 128) {
          uint2 vv;
          lds_u32x2(adr, vv);
          v4[0] = bf_lo(vv.x);
          v4[1] = bf_hi(vv.x);
          v4[2] = bf_lo(vv.y);
          v4[3] = bf_hi(vv.y);
        } else {
          uint4 vv;
          lds_u32x4(adr, vv);
          unpack8(vv, v4);
        }
      };
      int i = a;
      while (ok && i < bl) {
        const int r = (int)((t0 + i) / kRunTokens - w0);
        if (!wait_unit(s, seq_base + nruns + r)) {
          ok = false;
          break;
        }
        const int64_t rs2 = (w0 + r) * kRunTokens > t0 ? (w0 + r) * kRunTokens : t0;
        const int64_t re2 = (w0 + r + 1) * kRunTokens - t0;
        const int seg = re2 < (int64_t)bl ? (int)re2 : bl;  // this run's tokens of the range: [i, seg)
        uint32_t vadr = smem_u32(s.ring) + s.desc_off[(seq_base + nruns + r) % kDesc] +
                        (uint32_t)(t0 + i - rs2) * (2 * D) + lane * (2 * DL);
        uint32_t padr = pbf_u + (uint32_t)i * 8;
        for (; i + 4 <= seg; i += 4) {
          uint2 pw[4];
          float v4[4][DL];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            lds_u32x2(padr + q * 8, pw[q]);
            v_load(vadr + q * (2 * D), v4[q]);
          }
#pragma unroll
          for (int q = 0; q < 4; q++) pv_token(pw[q], v4[q]);
          vadr += 4 * (2 * D);
          padr += 32;
        }
        for (; i < seg; i++) {
          uint2 pw;
          float v4[DL];
          lds_u32x2(padr, pw);
          v_load(vadr, v4);
          pv_token(pw, v4);
          vadr += 2 * D;
          padr += 8;
        }
      }
      if (ok && has_pos) {
        const uint2 pw = pbf[b - 1];
        float v4[DL];
        v_load(smem_u32(s.scratch + kKvNewOff) + 2 * D + lane * (2 * DL), v4);
        pv_token(pw, v4);
      }
      if (ok) release_runs(s, seq_base + nruns, r0, r1, t0, t1, w0, C, lane);  // V runs
      cstamp(tr, 15);
    }
  }
  if (!ok) raise_abort(P, s, SPARK_ERR_LAUNCH);  // (skip the work, keep the barriers)
  consumer_bar();  // every warp is done with the scores and P
  cstamp(tr, 16);
  if (tr) tr[4] = gtimer();
  // ---- merge the ranges: O_w [kWarps][4][128] (one 128-dim half at a time), m_w, l_w
  float* ow = reinterpret_cast<float*>(s.scratch);
  float* mlw = ow + kWarps * 4 * 128;  // m [kWarps][4], l [kWarps][4]
  float* fac = mlw + 2 * kWarps * 4;   // f [4][kWarps], L [4], M [4]
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < 4; h++) {
      mlw[warp * 4 + h] = mx[h];
      mlw[kWarps * 4 + warp * 4 + h] = l[h];
    }
  }
#pragma unroll 1
  for (int ph = 0; ph < D / 128; ph++) {
    if (D == 128 || (lane >> 4) == ph) {
#pragma unroll
      for (int h = 0; h < 4; h++) {
        float* dst = ow + (warp * 4 + h) * 128 + DL * (D == 128 ? lane : (lane & 15));
#pragma unroll
        for (int d = 0; d < DL; d += 4)
          *reinterpret_cast<float4*>(dst + d) = make_float4(acc[h][d], acc[h][d + 1], acc[h][d + 2], acc[h][d + 3]);
      }
    }
    consumer_bar();
    if (ph == 0 && warp < 4) {  // warp h: M, the range factors (lane w), L in range order
      const int h = warp;
      const float mw = lane < kWarps ? mlw[lane * 4 + h] : ninf;
      const float lw = lane < kWarps ? mlw[kWarps * 4 + lane * 4 + h] : 0.0f;
      float M = mw;
#pragma unroll
      for (int off = 16; off >= 1; off /= 2) {
        const float o = __shfl_xor_sync(0xffffffffu, M, off);
        M = o > M ? o : M;
      }
      const float f = (mw == ninf || M == ninf) ? 0.0f : spark_exp_neg(__fsub_rn(mw, M));
      if (lane < kWarps) fac[h * kWarps + lane] = f;
      const float fl = __fmul_rn(f, lw);
      float fls[kWarps];
#pragma unroll
      for (int w = 0; w < kWarps; w++) fls[w] = __shfl_sync(0xffffffffu, fl, w);
      float L = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; w++) L = __fadd_rn(L, fls[w]);
      if (lane == 0) {
        fac[4 * kWarps + h] = L;
        fac[4 * kWarps + 4 + h] = M;
      }
    }
    if (ph == 0) consumer_bar();
    if (ph == 0) cstamp(tr, 17);
    for (int o = tid; o < 4 * 128; o += kConsumers) {
      const int h = o >> 7, d = o & 127;
      float v = 0.0f;
      if (fac[4 * kWarps + 4 + h] != ninf) {
        float O = 0.0f;
        for (int w = 0; w < kWarps; w++) O = __fadd_rn(O, __fmul_rn(fac[h * kWarps + w], ow[(w * 4 + h) * 128 + d]));
        v = __fdiv_rn(O, fac[4 * kWarps + h]);
      }
      part_o[((size_t)j * nq + 4 * g + h) * D + 128 * ph + d] = v;
    }
    if (ph + 1 < D / 128) consumer_bar();  // the first half's reads before the second half's writes
  }
  if (tid < 4) {
    const float M = fac[4 * kWarps + 4 + tid];
    part_lse[(size_t)j * nq + 4 * g + tid] = M == ninf ? ninf : __fadd_rn(spark_log(fac[4 * kWarps + tid]), M);
  }
  if (tr) tr[5] = gtimer();
  seq_base += 2 * nruns;
  return true;
}


// All 4 x D combined outputs of kv head g from its S published partials (the oracle's
// combine order).  The partials come into the scratch with 16-byte asynchronous copies,
// kCombineBytes / (16 D) splits per round, while the lse values load; each thread then
// accumulates its outputs over the splits in ascending order.  ToSmem: the outputs become
// the staged (fixed-point digit) input of the following SPARK_PRO_ATTN o_proj stage; else
// they go to attn_out.
template <int D, bool Spark, bool ToSmem, int NB = 1>
__device__ __forceinline__ void attn_combine_all(const SparkStage& st, const Smem& s, int tid, int g,
                                                 unsigned long long* tr, int bq = 0) {
  const int warp = tid >> 5, lane = tid & 31;
  cstamp(tr, 18);
  const int nq = st.nq, S = st.splits;
  constexpr int NO = (4 * D + kConsumers - 1) / kConsumers;  // outputs per thread
  constexpr int PER = kCombineBytes / (16 * D);              // splits per round
  constexpr int CH = D;                                      // 16-byte chunks per split (4 D floats)
  const float ninf = __int_as_float(0xff800000);
  const float* part_o = st.part_o + (NB > 1 ? (size_t)bq * S * nq * D : 0);
  const float* part_lse = st.part_lse + (NB > 1 ? (size_t)bq * S * nq : 0);
  const float* pc = reinterpret_cast<const float*>(s.scratch);             // [PER][4 D]
  float* lse_s = reinterpret_cast<float*>(s.scratch + kCombineLseOff);      // [4][S]
  float* w_s = lse_s + 4 * S;                                               // [4][S]
  float* mx_s = w_s + 4 * S;                                                // [4]
  const uint32_t pc_u = smem_u32(s.scratch);
  auto fetch = [&](int s0) {  // splits s0 .. s0 + PER - 1 into the round buffer
    const int ns = S - s0 < PER ? S - s0 : PER;
    for (int c = tid; c < ns * CH; c += kConsumers) {
      const int sp = c / CH, q = c - sp * CH;
      cp_async16(pc_u + (uint32_t)(sp * CH + q) * 16, part_o + ((size_t)(s0 + sp) * nq + 4 * g) * D + 4 * q);
    }
  };
  // the first round's partials stay in flight while the weights are computed from the lse
  fetch(0);
  for (int i = tid; i < 4 * S; i += kConsumers) {
    const int h = i / S, sp = i - h * S;
    lse_s[i] = __ldcg(part_lse + (size_t)sp * nq + 4 * g + h);
  }
  consumer_bar();
  cstamp(tr, 19);
  if (warp < 4) {  // warp h: max, exp, the sequential denominator and w / den of head h
    const int h = warp;
    float m = ninf;
    for (int sp = lane; sp < S; sp += 32) m = lse_s[h * S + sp] > m ? lse_s[h * S + sp] : m;
#pragma unroll
    for (int off = 16; off >= 1; off /= 2) {
      const float o2 = __shfl_xor_sync(0xffffffffu, m, off);
      m = o2 > m ? o2 : m;
    }
    for (int sp = lane; sp < S; sp += 32) {
      const float v = lse_s[h * S + sp];
      w_s[h * S + sp] = v == ninf ? 0.0f : spark_exp_neg(__fsub_rn(v, m));
    }
    __syncwarp();
    // den = sum of w_s in split order: batches of 8 loads ahead of the ordered adds
    float den = 0.0f;
    for (int s0 = 0; s0 < S; s0 += 8) {
      float w8[8];
#pragma unroll
      for (int q = 0; q < 8; q++) w8[q] = s0 + q < S ? w_s[h * S + s0 + q] : 0.0f;
#pragma unroll
      for (int q = 0; q < 8; q++)
        if (s0 + q < S) den = __fadd_rn(den, w8[q]);
    }
    __syncwarp();
    for (int sp = lane; sp < S; sp += 32) w_s[h * S + sp] = __fdiv_rn(w_s[h * S + sp], den);
    if (lane == 0) mx_s[h] = m;
  }
  cp_async_wait_all();
  consumer_bar();  // the weights and the first round's partials
  cstamp(tr, 20);
  float a[NO];
#pragma unroll
  for (int k = 0; k < NO; k++) a[k] = 0.0f;
#pragma unroll 1
  for (int s0 = 0; s0 < S; s0 += PER) {
    if (s0 > 0) {  // the next round's partials (the previous round's reads are done)
      consumer_bar();
      fetch(s0);
      cp_async_wait_all();
      consumer_bar();
    }
    const int ns = S - s0 < PER ? S - s0 : PER;
#pragma unroll
    for (int k = 0; k < NO; k++) {
      const int o = tid + k * kConsumers;
      if (o < 4 * D) {
        const int h = o / D;
        for (int b0 = 0; b0 < ns; b0 += 6) {  // 6 splits' loads ahead of their ordered adds
          float wv[6], pv[6];
          bool live[6];
#pragma unroll
          for (int q = 0; q < 6; q++) {
            const int sp = b0 + q;
            live[q] = sp < ns && lse_s[h * S + s0 + sp] != ninf;
            wv[q] = sp < ns ? w_s[h * S + s0 + sp] : 0.0f;
            pv[q] = sp < ns ? pc[sp * 4 * D + o] : 0.0f;
          }
#pragma unroll
          for (int q = 0; q < 6; q++)
            if (live[q]) a[k] = __fadd_rn(a[k], __fmul_rn(wv[q], pv[q]));
        }
      }
    }
  }
  cstamp(tr, 21);
  if constexpr (ToSmem) consumer_bar();  // the last round's reads before xin overwrites the round buffer
  uint16_t* xin = reinterpret_cast<uint16_t*>(s.scratch + kXinOff);  // [4 D]
#pragma unroll
  for (int k = 0; k < NO; k++) {
    const int o = tid + k * kConsumers;
    if (o < 4 * D) {
      const int h = o / D;
      uint16_t ob = f2bf(mx_s[h] != ninf ? a[k] : 0.0f);
      if constexpr (Spark) {
        if (st.gate)  // headwise output gate (written by the qkv stage)
          ob = f2bf(__fmul_rn(bf2f(ob), bf2f(__ldcg(static_cast<const unsigned short*>(st.gate) + 4 * g + h))));
      }
      if constexpr (ToSmem) {
        xin[o] = ob;
      } else {
        static_cast<uint16_t*>(st.attn_out)[((NB > 1 ? (size_t)bq * nq : 0) + (size_t)4 * g) * D + o] = ob;
      }
    }
  }
  if constexpr (ToSmem) {  // stage the 4 D values as the o_proj K part's fixed-point digits
    consumer_bar();
    constexpr int NG = 4 * D / 8;  // 8-element groups: threads 0 .. NG - 1 (whole warps)
    if (tid < NG) {
      float v[8];
      unpack8(*reinterpret_cast<const uint4*>(xin + 8 * tid), v);
      stage_group(v, true, tid, reinterpret_cast<uint32_t*>(s.scratch),
                  reinterpret_cast<int2*>(s.scratch + 64 * (4 * D / 32)));
    }
  }
  cstamp(tr, 22);
}

// Waits (bounded) until all S splits of kv head g have published in this launch.
__device__ __forceinline__ bool attn_wait_head(const StepParams& P, const SparkStage& st, const Smem& s, int g) {
  const int target = st.splits * (int)(s.misc64[2] + 1);
  const unsigned long long tw = gtimer();
  while (ld_acquire(st.head_counters + g) < target)
    if (*s.abort_flag || gtimer() - tw > kWaitNs) return false;
  return true;
}

// Tasks (kv head g, split j) = t / S, t % S go round-robin to the CTAs (t = cta, cta +
// CTAs, ...).  Fused (the next stage is a SPARK_PRO_ATTN o_proj; one task per CTA): each
// CTA publishes its split, waits for the head's other splits and combines the whole head
// into shared memory.  Otherwise each split counts itself on the head's counter with an
// acquire-release add and the one that completes the head combines it into attn_out,
// so no CTA waits for another (several tasks per CTA cannot deadlock).  !Multi: at most
// one task per CTA, in a form with no loop state (the usual program; a loop here costs
// the GEMV stages registers in the same kernel).
// NB > 1: tasks (sequence b, kv head g, split j) = t / (nkv S), ..., never fused (the
// host checks), each sequence's heads counted on its own counters.
template <int D, bool Multi, bool Spark, int NB = 1>
__device__ __forceinline__ bool attn_stage_d(const StepParams& P, const SparkStage& st, const Smem& s,
                                          uint32_t& seq_base, int tid, bool fused) {
  const int S = st.splits, ntask = NB * st.nkv * S;
  unsigned long long* tr = (tid == 0 && P.io.trace)
                               ? P.io.trace + ((size_t)blockIdx.x * P.num_stages + s.flag[2]) * kTraceSlots
                               : nullptr;
  auto finish = [&](int g) {
    consumer_bar();  // the split's partials (all threads) before its count
    if (fused) {
      if (tid == 0) {
        asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(st.head_counters + g) : "memory");
        if (!attn_wait_head(P, st, s, g)) raise_abort(P, s, SPARK_ERR_LAUNCH);
        if (tr) tr[6] = gtimer();
      }
      consumer_bar();
      attn_combine_all<D, Spark, true>(st, s, tid, g, tr);
    } else {
      if (tid == 0) {
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(st.head_counters + g) : "memory");
        s.flag[3] = old == st.splits * (int)(s.misc64[2] + 1) - 1;
        if (tr) tr[6] = gtimer();
      }
      consumer_bar();
      if (s.flag[3]) attn_combine_all<D, Spark, false>(st, s, tid, g, tr);
    }
    if (tr) tr[7] = gtimer();
  };
  if constexpr (NB > 1) {
    const int per = st.nkv * S;
#pragma unroll 1
    for (int t = blockIdx.x; t < ntask; t += gridDim.x) {
      const int bq = t / per, tb = t - bq * per, g = tb / S;
      if (!attn_split<D, Spark, NB>(P, st, s, seq_base, tid, g, tb - g * S, bq)) return false;
      consumer_bar();  // the split's partials (all threads) before its count
      if (tid == 0) {
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                     : "=r"(old)
                     : "l"(st.head_counters + (size_t)bq * st.nkv + g)
                     : "memory");
        s.flag[3] = old == st.splits * (int)(s.misc64[2] + 1) - 1;
      }
      consumer_bar();
      if (s.flag[3]) attn_combine_all<D, Spark, false, NB>(st, s, tid, g, tr, bq);
      if (t + (int)gridDim.x < ntask) consumer_bar();  // this task's shared memory before the next task's
    }
  } else if constexpr (!Multi) {
    if ((int)blockIdx.x >= ntask) return true;
    const int g = blockIdx.x / S, j = blockIdx.x - g * S;
    if (!attn_split<D, Spark>(P, st, s, seq_base, tid, g, j)) return false;
    finish(g);
  } else {
#pragma unroll 1
    for (int t = blockIdx.x; t < ntask; t += gridDim.x) {
      if (!attn_split<D, Spark>(P, st, s, seq_base, tid, t / S, t - (t / S) * S)) return false;
      finish(t / S);
      if (t + (int)gridDim.x < ntask) consumer_bar();  // this task's shared memory before the next task's
    }
  }
  return true;
}

// head_dim 256 in the Spark instantiation, 128 in the others (the host checks; one
// attention body per kernel keeps its registers)
template <bool Multi, bool Spark, int NB = 1>
__device__ __forceinline__ bool attn_stage(const StepParams& P, const SparkStage& st, const Smem& s, uint32_t& seq_base,
                                        int tid, bool fused) {
  if constexpr (NB > 1) {
    return attn_stage_d<128, true, false, NB>(P, st, s, seq_base, tid, false);
  } else if constexpr (Spark) {
    return attn_stage_d<256, Multi, true>(P, st, s, seq_base, tid, fused);
  } else {
    return attn_stage_d<128, Multi, false>(P, st, s, seq_base, tid, fused);
  }
}

// ------------------------------------------------------------------ the kernel
__device__ __forceinline__ bool wait_stage(const StepParams& P, const Smem& s, int idx) {
  const int* ctr = P.io.counters + idx;
  const SparkStage& w = stage_at(P, idx);
  const int target = stage_target(P.io, w, (int)gridDim.x, s.misc64[2]);
  // an exchange stage is counted by other GPUs: acquire at system scope
  const bool sys = w.xchg != 0;
  auto poll = [&]() { return reached(sys ? ld_acquire_sys(ctr) : ld_acquire(ctr), target); };
  if (poll()) return true;
  const unsigned long long t0 = gtimer();
  for (;;) {  // each poll is one L2 round trip: spin without sleeping
    if (poll()) return true;
    if (ld_acquire(P.io.counters + P.num_stages + 1)) return false;
    if (gtimer() - t0 > kWaitNs) return false;
  }
}

// Q6: the program has Q6_K GEMV stages; Multi: an attention stage has more tasks than
// CTAs; Spark: the program uses a Spark layer feature (head_dim 256, sliding window,
// output gate, partial RoPE, GELU * mul); NB: sequences decoded together (batch
// programs: Q4_0, head_dim 128, one GPU, any number of attention tasks).  Each is its
// own instantiation so the usual program (Q4_0, one attention task per CTA, one
// sequence) carries none of their registers.
template <bool Q6, bool Multi, bool Spark, bool TP, int NB = 1>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const StepParams P) {
  static_assert(NB == 1 || (!Q6 && !Spark && !TP), "batch programs: Q4_0, head_dim 128, one GPU");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const Smem s = carve<NB>(smem_raw);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < kDesc; i++) {
      mbar_init(smem_u32(s.full + i), 1);
      mbar_init(smem_u32(s.empty + i), 1);
      s.done[i] = 0;
      s.desc_seq[i] = 0xffffffffu;  // no copy issued yet
    }
    *s.abort_flag = 0;
    s.misc64[2] = P.io.counters[P.num_stages + 2];  // launch generation (attention head counters)
    s.misc64[3] = 0;                                 // no cached launch constants yet
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (tid >= kConsumers) {
    if (tid == kConsumers) {
      Producer<NB> pr(P, s);
      pr.template run<NB == 1 ? Multi : true, Spark>();
    }
    return;
  }
  uint32_t seq_base = 0;
  for (int i = 0; i < P.num_stages; i++) {
    if (tid < kStageWords)  // 8-byte pieces: the inline stage in the launch parameters is only 8-byte aligned
      reinterpret_cast<unsigned long long*>(s.stage)[tid] =
          reinterpret_cast<const unsigned long long*>(&stage_at(P, i))[tid];
    unsigned long long* tr = P.io.trace ? P.io.trace + ((size_t)blockIdx.x * P.num_stages + i) * kTraceSlots : nullptr;
    if (tid == 0 && tr) tr[0] = gtimer();
    if (tid == 0) s.flag[2] = i;  // stage index for the stage functions' trace stamps
    {
      // values that are fixed for the whole launch (position, block table, RoPE table):
      // fetched before the stage barrier so their latency hides behind it
      const SparkStage& nx = stage_at(P, i);
      const bool gemv = nx.kind == SPARK_STAGE_GEMV || nx.kind == SPARK_STAGE_GEMV_Q6;
      const bool rope = gemv && nx.epi == SPARK_EPI_ROPE_KV;
      if (gemv && nx.norm) {  // RMSNorm weight (a constant) next to the staging area
        const uint4* src = static_cast<const uint4*>(nx.gamma);
        uint4* dst = reinterpret_cast<uint4*>(s.scratch + (NB == 1 ? 72 * (nx.k >> 5) + 4 * nx.k : 4 * nx.k * NB));
        for (int q = tid; q < (nx.k >> 3); q += kConsumers) dst[q] = __ldg(src + q);
      }
      if (tid == 32) {  // touch the stage's activation buffers (value unused) to warm their translations
        const void* bufs[8] = {nx.a, nx.b, nx.out, nx.res_out, nx.q, nx.kv_new, nx.part_o, nx.attn_out};
#pragma unroll
        for (int b2 = 0; b2 < 8; b2++)
          if (bufs[b2]) asm volatile("prefetch.global.L2 [%0];" ::"l"(bufs[b2]));
      }
      // the same position / RoPE row serve every layer: fetch them once per launch
      // (Spark: sliding and full layers rotate with different tables, so the table is part
      // of the key and a layer of the other type fetches its own row)
      const long long key = (long long)reinterpret_cast<uintptr_t>(nx.pos) ^
                            (Spark && rope ? (long long)reinterpret_cast<uintptr_t>(nx.cos_sin) : 0ll);
      if (NB > 1 && (rope || nx.kind == SPARK_STAGE_ATTN) && s.misc64[3] != key && tid < 32) {
        // the NB sequences' positions, cache offsets of the decoded tokens and RoPE rows
        if (tid < NB) {
          const int64_t pos = __ldcg(nx.pos + tid);
          s.bpos[tid] = pos;
          if (rope) {
            const int64_t blk = pos / nx.block_size, off = pos - blk * nx.block_size;
            s.bkvoff[tid] =
                ((int64_t)nx.block_table[(size_t)tid * nx.bt_stride + blk] * nx.nkv * nx.block_size + off) * 128;
          }
        }
        __syncwarp();
        if (rope)
          for (int e = tid; e < NB * 128; e += 32)
            s.rope_cs[e] = static_cast<const uint16_t*>(nx.cos_sin)[(size_t)s.bpos[e >> 7] * 128 + (e & 127)];
        __syncwarp();
        if (rope && tid == 0) s.misc64[3] = key;
      } else if (NB == 1 && (rope || nx.kind == SPARK_STAGE_ATTN) && s.misc64[3] != key && tid < 32) {
        const int64_t pos = __ldcg(nx.pos);
        if (tid == 0) {
          s.misc64[0] = pos;
          if (rope) {
            const int64_t blk = pos / nx.block_size, off = pos - blk * nx.block_size;
            s.misc64[1] = ((int64_t)nx.block_table[blk] * nx.nkv * nx.block_size + off) * nx.head_dim;
          }
        }
        if (rope) {  // a row of r = rotary dims (Spark partial RoPE) or head_dim entries
          const int r = Spark && nx.rotary_dim ? nx.rotary_dim : nx.head_dim;
          const uint16_t* cs = static_cast<const uint16_t*>(nx.cos_sin) + (size_t)pos * r;
          for (int d = tid; d < r; d += 32) s.rope_cs[d] = cs[d];
        }
        __syncwarp();
        if (rope && tid == 0) s.misc64[3] = key;  // cached only once the RoPE row is in place
      }
    }
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
    if (tid == 0 && tr) tr[1] = gtimer();
    const SparkStage& st = *s.stage;
    // an attention stage followed by a SPARK_PRO_ATTN o_proj combines into shared memory
    // and is waited on by no stage (the host checks): it is not counted
    const bool fused = st.kind == SPARK_STAGE_ATTN && i + 1 < P.num_stages && stage_at(P, i + 1).pro == SPARK_PRO_ATTN;
    // both stage functions keep every consumer on the same barriers; a stage that
    // fails returns false in all threads (attention: a split longer than the scratch)
    bool ok;
    if constexpr (NB > 1)
      ok = st.kind != SPARK_STAGE_ATTN ? gemv_stage_b<NB>(P, st, s, seq_base, tid)
                                       : attn_stage<true, false, NB>(P, st, s, seq_base, tid, false);
    else
      ok = st.kind != SPARK_STAGE_ATTN ? gemv_stage<Q6, Spark, TP>(P, st, s, seq_base, tid)
                                       : attn_stage<Multi, Spark>(P, st, s, seq_base, tid, fused);
    consumer_bar();
    if (!ok) return;
    if (tid == 0 && tr) tr[2] = gtimer();
    // a tagged exchange stage is not counted (its readers wait on its words); a fused
    // attention stage neither
    if (tid == 0 && !*s.abort_flag && !fused && st.xchg != SPARK_XCHG_TAGGED) {  // release: the CTA's writes
                                                                                 // (ordered by the barrier) first
      if (st.xchg) {  // writes to every rank's window, then a count on every rank
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int p = 0; p < P.io.tp_size; p++)
          asm volatile("red.relaxed.sys.global.add.s32 [%0], 1;" ::"l"(peer_addr(P.io, p, P.io.counters + i))
                       : "memory");
      } else {
        asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(P.io.counters + i) : "memory");
      }
    }
  }
  // ---- the last CTA to finish turns the argmax into a token and resets the counters
  // (tensor parallel: counts launches instead of resetting; the key is complete once
  // every rank's CTAs have counted the last stage)
  if (tid == 0 && !*s.abort_flag) {
    __threadfence();
    const SparkStepIO& io = P.io;
    const int ncta = (int)gridDim.x;
    const bool tp = io.tp_size > 1;
    const int done = atomicAdd(io.counters + P.num_stages, 1);
    const int last_done = tp ? (int)((unsigned)ncta * (unsigned)(s.misc64[2] + 1) - 1u) : ncta - 1;
    if (done == last_done) {
      __threadfence();
      bool ok = true;
      if (tp) {
        const int li = P.num_stages - 1;
        const SparkStage& ls = stage_at(P, li);
        const int target = stage_target(io, ls, ncta, s.misc64[2]);
        const unsigned long long t0 = gtimer();
        while (!reached(ls.xchg ? ld_acquire_sys(io.counters + li) : ld_acquire(io.counters + li), target)) {
          if (gtimer() - t0 > kWaitNs) {
            ok = false;
            break;
          }
        }
        if (!ok) raise_abort(P, s, SPARK_ERR_LAUNCH);
      }
      if (ok) {
        if (io.key) {
#pragma unroll 1
          for (int b = 0; b < NB; b++) {  // sequence b's token
            const unsigned long long k = atomicAdd(io.key + b, 0ull);
            const int32_t tok = (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
            if (io.token_out) io.token_out[b] = tok;
            if (io.token_log) io.token_log[(io.step ? io.step[0] : 0) * NB + b] = tok;
            io.key[b] = 0ull;
          }
        }
        if (io.step) io.step[0] += 1;
        if (io.pos)
#pragma unroll 1
          for (int b = 0; b < NB; b++) io.pos[b] += 1;
        if (!tp)
          for (int i = 0; i <= P.num_stages; i++) io.counters[i] = 0;
        io.counters[P.num_stages + 2] += 1;  // next launch's generation
        __threadfence();
      }
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
    const int ra = t16_row_x(rowmap, rg, g, n, aux), rb = t16_row_x(rowmap, rg, g + 8, n, aux);
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

// ------------------------------------------------------------------ T6 packing (Q6_K)
__device__ __forceinline__ int q6k_code_dev(const uint8_t* blk, int e) {  // q + 32 of weight e
  const int h = e >> 7, l = e & 127;
  const int lo = (blk[64 * h + (l & 63)] >> (4 * (l >> 6))) & 15;
  const int hi = (blk[128 + 32 * h + (l & 31)] >> (2 * (l >> 5))) & 3;
  return lo | (hi << 4);
}

// blocks: gguf Q6_K rows [n][k / 256 * 210]; one thread per (unit, 64-weight group, lane)
__global__ void t6_pack_kernel(const uint8_t* __restrict__ blocks, int n, int k, int kp, uint8_t* __restrict__ out) {
  const int Kp = k / kp, groups = Kp >> 6;
  const size_t row_bytes = (size_t)(k >> 8) * 210;
  const size_t total = (size_t)(n >> 4) * kp * groups * 32;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int L = (int)(i & 31);
    const size_t gi = i >> 5;
    const int G = (int)(gi % groups);
    const int u = (int)(gi / groups);
    const int rg = u / kp, kpi = u - rg * kp;
    const int g = L >> 2, c = L & 3;
    const int ra = 16 * rg + g, rb = ra + 8;
    const uint8_t* rowa = blocks + (size_t)ra * row_bytes;
    const uint8_t* rowb = blocks + (size_t)rb * row_bytes;
    uint8_t* unit = out + (size_t)u * t6_unit_bytes(Kp);
    uint8_t* grp = unit + Kp / 8 + Kp + (size_t)G * 768;
    uint32_t nibw[4], hw[2];
#pragma unroll
    for (int j = 0; j < 2; j++) {  // the two 32-weight tiles of the group
      uint32_t n0 = 0, n1 = 0, h = 0;
#pragma unroll
      for (int b = 0; b < 4; b++) {
        const int e0 = kpi * Kp + 64 * G + 32 * j + 4 * c + b;  // k = 4c + b (sub-block 0)
        const int e2 = e0 + 16;                                  // k = 16 + 4c + b (sub-block 1)
        const int qa0 = q6k_code_dev(rowa + (size_t)(e0 >> 8) * 210, e0 & 255);
        const int qa2 = q6k_code_dev(rowa + (size_t)(e2 >> 8) * 210, e2 & 255);
        const int qb0 = q6k_code_dev(rowb + (size_t)(e0 >> 8) * 210, e0 & 255);
        const int qb2 = q6k_code_dev(rowb + (size_t)(e2 >> 8) * 210, e2 & 255);
        n0 |= (uint32_t)((qa0 & 15) | ((qa2 & 15) << 4)) << (8 * b);
        n1 |= (uint32_t)((qb0 & 15) | ((qb2 & 15) << 4)) << (8 * b);
        h |= (uint32_t)((qa0 >> 4) | ((qb0 >> 4) << 2) | ((qa2 >> 4) << 4) | ((qb2 >> 4) << 6)) << (8 * b);
      }
      nibw[2 * j] = n0;
      nibw[2 * j + 1] = n1;
      hw[j] = h;
    }
    *reinterpret_cast<uint4*>(grp + 16 * L) = make_uint4(nibw[0], nibw[1], nibw[2], nibw[3]);
    *reinterpret_cast<uint2*>(grp + 512 + 8 * L) = make_uint2(hw[0], hw[1]);
    if (c == 0) {  // the group's 4 sub-block scales and (every 4 groups) the super-block d of rows ra, rb
      const int e = kpi * Kp + 64 * G;
      const uint8_t* ba = rowa + (size_t)(e >> 8) * 210;
      const uint8_t* bb = rowb + (size_t)(e >> 8) * 210;
#pragma unroll
      for (int sbk = 0; sbk < 4; sbk++) {
        const int s16 = ((e & 255) >> 4) + sbk;  // sub-block within the super-block
        uint8_t* sc = unit + Kp / 8 + (size_t)(4 * G + sbk) * 16 + 2 * g;
        sc[0] = ba[192 + s16];
        sc[1] = bb[192 + s16];
      }
      if ((G & 3) == 0) {
        uint8_t* dp = unit + (size_t)(G >> 2) * 32 + 4 * g;
        dp[0] = ba[208];
        dp[1] = ba[209];
        dp[2] = bb[208];
        dp[3] = bb[209];
      }
    }
  }
}

// gguf Q6_K blocks -> fp32 weights, the decode of orc_q6k_dequantize (validation)
__global__ void q6k_dequant_kernel(const uint8_t* __restrict__ blocks, int64_t nblocks, float* __restrict__ w) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nblocks * 256;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t* blk = blocks + (i >> 8) * 210;
    const int e = (int)(i & 255);
    const float d = h2f((uint16_t)(blk[208] | (blk[209] << 8)));
    const float sc = __fmul_rn(d, (float)(int8_t)blk[192 + (e >> 4)]);
    w[i] = __fmul_rn(sc, (float)(q6k_code_dev(blk, e) - 32));
  }
}

}  // namespace step
}  // namespace spark
