// Tensor-core Q4_0 GEMM for prompt prefill: Y[t][n] = bf16(sum_k W[n][k] X[t][k]).
//
// The reference's prefill multiplies the chunk's activations by the bf16 dequantization
// of each Q4_0 weight (integration/weights.py:28-31 `dequantize(...).bfloat16()`, then
// vLLM's torch matmul).  This kernel does the same product without a bf16 copy of the
// weights in HBM: each CTA dequantizes its 128-row weight tile straight into shared
// memory (w = bf16(fp32(d) * (q - 8)), the same rounding as spark_q4_dequantize_bf16),
// stages 128 tokens of X beside it, and one thread issues tcgen05.mma (kind::f16, bf16
// operands, fp32 accumulators in tensor memory).
//
// Tile: M = 128 weight rows (TMEM lanes), N = 128 tokens (TMEM columns), K = 64 per
// stage (one 128-byte swizzle atom of bf16), 2 stages; 256 threads, two per tile row
// (one per 32-wide half of a K step).  Both operands are K-major with the 128-byte
// swizzle: row r of a tile at (r / 8) * 1024 + (r % 8) * 128, its 16-byte chunk c at
// chunk position c ^ (r % 8).
//
// Waits on the MMA completion barriers are bounded by %globaltimer (limit_ns, a kernel
// argument).  A wait that runs out sets *error = 1; the CTA then waits, with its own
// bound of kDrainNs, for the commit of the last step whose MMAs it issued (a commit
// tracks every earlier MMA of the issuing thread), so no MMA still reads the shared
// tiles or writes the accumulator columns when the CTA frees them.  If that drain also
// runs out, the CTA sets *error = 2 and exits WITHOUT freeing its tensor memory: the
// context must then be treated as unusable.  tcgen05.alloc itself has no bound: it
// blocks until 128 columns are free, so the kernel assumes no other tensor-memory user
// on the SM at the same time (shared memory admits at most 3 of its own CTAs per SM,
// 384 of the 512 columns).
#pragma once

#include <cstdint>

#include "common.cuh"

namespace spark {
namespace tc {

constexpr int kBM = 128;                  // weight rows per tile (MMA M)
constexpr int kBN = 128;                  // tokens per tile (MMA N)
constexpr int kBK = 64;                   // K per stage
constexpr int kStages = 2;
constexpr int kThreads = 256;            // two threads per tile row: one per half of a K step
constexpr int kTileBytes = kBM * kBK * 2;  // 16 KB; the token tile is the same size (kBN == kBM)
constexpr int kSmemBytes = kStages * 2 * kTileBytes + 1024 + 64;  // tiles, 1024-B alignment slack, barriers
constexpr unsigned long long kWaitNs = 500ull * 1000 * 1000;      // default limit of a wait: 0.5 s
constexpr unsigned long long kDrainNs = 2000ull * 1000 * 1000;    // drain of issued MMAs after a timeout

static_assert(kBN == kBM, "token and weight tiles share one size");

// instruction descriptor (kind::f16): fp32 D (bits 4-5 = 1), bf16 A (bits 7-9 = 1) and
// B (bits 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                            ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// shared-memory matrix descriptor of a K-major 128-byte-swizzled tile at `addr`
// (1024-byte aligned): start >> 4, leading offset 16 B (unused with this swizzle),
// 8-row groups 1024 B apart, descriptor version 1, layout SWIZZLE_128B (2)
__device__ __forceinline__ uint64_t sdesc(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// non-blocking test of the phase, so a limit of 0 ns gives up after one look
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, unsigned long long limit_ns) {
  const unsigned long long t0 = now_ns();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{.reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p;}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (now_ns() - t0 >= limit_ns) return false;
  }
}

// 8 weights of one Q4_0 block as 4 bf16 pairs: the nibbles at `shift` of the 8 bytes
// held by (w0, w1).  q - 8 as fp32 from the bits of 2^23 + q minus 2^23 + 8 (exact);
// fp32(d) * (q - 8) is exact in fp32 (11 + 4 significant bits), and cvt.rn.bf16x2 rounds
// the pair to nearest-even (NaN -> 0x7fff), the same bits as f2bf.
__device__ __forceinline__ uint4 deq8(uint32_t w0, uint32_t w1, int shift, float s) {
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const uint32_t wd = i < 2 ? w0 : w1;
    const int b = (2 * i) & 3;
    const float m0 = __uint_as_float(0x4B000000u | ((wd >> (8 * b + shift)) & 15u)) - 8388616.0f;
    const float m1 = __uint_as_float(0x4B000000u | ((wd >> (8 * (b + 1) + shift)) & 15u)) - 8388616.0f;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(o[i]) : "f"(__fmul_rn(s, m1)), "f"(__fmul_rn(s, m0)));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// global loads of half a K step for this thread (half h = 0 / 1: k 32h .. 32h + 31 of
// the step): its weight row's Q4_0 block and its token row's 32 activations (zeros past
// the last row / token)
__device__ __forceinline__ void load_step(const uint8_t* qrow, const uint16_t* drow, const uint16_t* xrow, bool nv,
                                          bool tv, int kb, int h, uint4& q, uint16_t& dd, uint4 (&xv)[4]) {
  const int bi = kb * 2 + h;
  dd = nv ? __ldg(drow + bi) : (uint16_t)0;
  q = nv ? __ldg(reinterpret_cast<const uint4*>(qrow + (size_t)bi * 16)) : make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int c = 0; c < 4; c++)
    xv[c] = tv ? __ldg(reinterpret_cast<const uint4*>(xrow + (size_t)kb * kBK + (4 * h + c) * 8))
               : make_uint4(0, 0, 0, 0);
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__global__ void __launch_bounds__(kThreads) q4_gemm_tc_kernel(const uint16_t* __restrict__ x,
                                                         const uint8_t* __restrict__ qs,
                                                         const uint16_t* __restrict__ d, uint16_t* __restrict__ y,
                                                         int T, int N, int K, int* __restrict__ error,
                                                         unsigned long long limit_ns) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = (uint32_t)__cvta_generic_to_shared(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t bars = base + kStages * 2 * kTileBytes;  // kStages mbarriers (8 B each)
  const uint32_t tslot = bars + 8 * kStages;               // tensor-memory base written by tcgen05.alloc
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kBM, t0 = blockIdx.y * kBN;
  const int nk = K / kBK, kblocks = K / 32;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kStages; s++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bars + 8 * s));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tslot), "r"(kBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  uint32_t tmem;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(tmem) : "r"(tslot) : "memory");

  const int r = tid & (kBM - 1), h = tid >> 7;  // tile row r, half h of each K step
  const int n = n0 + r, t = t0 + r;              // this thread stages weight row n and token row t
  const uint8_t* qrow = qs + (size_t)(n < N ? n : 0) * (K / 2);
  const uint16_t* drow = d + (size_t)(n < N ? n : 0) * kblocks;
  const uint16_t* xrow = x + (size_t)(t < T ? t : 0) * K;
  const bool nv = n < N, tv = t < T;
  // software pipeline: two register sets alternate, so step kb + 2's global loads are
  // in flight while steps kb and kb + 1 are dequantized into shared memory and multiplied
  uint4 qa, xa[4], qb, xb[4];
  uint16_t da, db;
  load_step(qrow, drow, xrow, nv, tv, 0, h, qa, da, xa);
  if (nk > 1) load_step(qrow, drow, xrow, nv, tv, 1, h, qb, db, xb);
  // one K step from register set (q, dd, xv), which is then refilled with step kb + 2;
  // false (in every thread) if the wait for the stage's previous MMAs ran out
  auto step = [&](int kb, uint4& q, uint16_t& dd, uint4 (&xv)[4]) -> bool {
    const int s = kb & 1;
    const uint4 qc = q;
    const uint16_t dc = dd;
    uint4 xc[4];
#pragma unroll
    for (int c = 0; c < 4; c++) xc[c] = xv[c];
    if (kb + 2 < nk) load_step(qrow, drow, xrow, nv, tv, kb + 2, h, q, dd, xv);
    if (kb >= kStages) {  // the MMAs of step kb - 2 read this stage
      const bool mine = bar_wait(bars + 8 * s, ((kb - kStages) >> 1) & 1, limit_ns);
      if (__syncthreads_or(!mine)) return false;
    }
    const uint32_t a_tile = base + s * 2 * kTileBytes, b_tile = a_tile + kTileBytes;
    {  // rows past N hold zero codes and scales: zero weights
      const float sc = h2f(dc);
      sts128(a_tile + sw128(r, 4 * h + 0), deq8(qc.x, qc.y, 0, sc));
      sts128(a_tile + sw128(r, 4 * h + 1), deq8(qc.z, qc.w, 0, sc));
      sts128(a_tile + sw128(r, 4 * h + 2), deq8(qc.x, qc.y, 4, sc));
      sts128(a_tile + sw128(r, 4 * h + 3), deq8(qc.z, qc.w, 4, sc));
    }
#pragma unroll
    for (int c = 0; c < 4; c++) sts128(b_tile + sw128(r, 4 * h + c), xc[c]);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint64_t ad = sdesc(a_tile), bd = sdesc(b_tile);
#pragma unroll
      for (int j = 0; j < kBK / 16; j++) {  // K = 16 per MMA: 32 bytes further along the swizzled rows
        const uint32_t acc = (kb | j) != 0;
        asm volatile(
            "{.reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;}" ::"r"(
                tmem),
            "l"(ad + 2 * j), "l"(bd + 2 * j), "r"(kIdesc), "r"(acc));
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bars + 8 * s)
                   : "memory");
    }
    return true;
  };
  bool ok = true;
  int issued = 0;  // steps whose MMAs and commit were issued
  for (int kb = 0; kb < nk && ok; kb += 2) {
    ok = step(kb, qa, da, xa);
    issued += ok;
    if (ok && kb + 1 < nk) {
      ok = step(kb + 1, qb, db, xb);
      issued += ok;
    }
  }
  if (ok) {  // the last commit tracks every MMA this CTA issued
    const bool mine = bar_wait(bars + 8 * ((nk - 1) & 1), ((nk - 1) >> 1) & 1, limit_ns);
    ok = !__syncthreads_or(!mine);
  }
  if (!ok) {
    // a wait ran out: report it, then wait (own bound) until every issued MMA has
    // completed before the shared tiles and the accumulator columns are given up
    if (tid == 0) atomicExch(error, 1);
    bool drained = true;
    if (issued > 0) {
      const int last = issued - 1;
      drained = !__syncthreads_or(!bar_wait(bars + 8 * (last & 1), (last >> 1) & 1, kDrainNs));
    }
    if (!drained) {  // MMAs still outstanding after kDrainNs: keep the columns, poison
      if (tid == 0) atomicExch(error, 2);
      return;
    }
  }
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (ok) {
    // TMEM lane = weight row (warp w reaches lanes 32 (w % 4) ..), columns = tokens:
    // warps 0-3 read columns [0, 64), warps 4-7 [64, 128)
    const int row = n0 + (warp & 3) * 32 + lane, cb = (warp >> 2) * (kBN / 2);
#pragma unroll 1
    for (int c0 = cb; c0 < cb + kBN / 2; c0 += 16) {
      uint32_t v[16];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)c0));
      asm volatile("tcgen05.wait::ld.sync.aligned;"
                   : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                     "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                     "+r"(v[15])
                   :
                   : "memory");
      if (row < N) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const int tt = t0 + c0 + i;
          if (tt < T) y[(size_t)tt * N + row] = f2bf(__uint_as_float(v[i]));
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBN));
  }
}

}  // namespace tc
}  // namespace spark
