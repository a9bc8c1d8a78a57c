// q4_gemv_ring.cuh -- persistent, warp-specialised Q4_0 GEMV with a TMA-bulk weight ring.
//
// Same arithmetic and order as q4_gemv.cuh (each row is split over the 16 lanes of
// a half warp, lane l owns blocks l, l+16, ... ascending; see that file), so the
// outputs are bit-identical to the register-direct kernel and to the CPU oracle.
// What changes is how the weights reach the SM:
//
//   * one CTA per SM (grid = number of SMs), 12 consumer warps + 1 producer warp; at
//     most 72 registers per thread (launch bounds of 2 CTAs per SM), so when the ring
//     fits half the shared memory (the single-op GEMV of 9728 x 2560, qkv, o_proj) the
//     next launch's CTA is resident beside this one and its producer streams weights
//     while this CTA finishes (back-to-back 9728 x 2560: 5.9 -> 5.0 us);
//   * the CTA owns a contiguous range of "units" (a unit is a row pair in pair mode,
//     one row in single mode); units are processed in rounds of up to 24 (one per
//     consumer half warp), each round in K-chunks of 16*CB blocks per row;
//   * the producer warp copies every (round, chunk) stage -- per row one bulk copy
//     of the nibble bytes and one of the fp16 scales -- with cp.async.bulk into a
//     ring of shared-memory slots guarded by mbarriers (full: transaction bytes,
//     empty: one arrival per consumer warp);
//   * the producer starts before griddepcontrol.wait: weights do not depend on the
//     previous kernel, so their fetch overlaps its tail and this kernel's prologue
//     (activation staging / RMSNorm), which only the consumers wait for.
//
// Every mbarrier wait is bounded; on a timeout the kernel records an error code in
// GemvArgs::error, the producer waits (bounded) for the copies it issued, and the
// CTA returns.
#pragma once

#include <type_traits>

#include "q4_gemv.cuh"

namespace spark {

constexpr int kRingConsumerWarps = 12;
constexpr int kRingThreads = (kRingConsumerWarps + 1) * 32;
constexpr int kRingUnitsPerRound = kRingConsumerWarps * 2;
constexpr uint32_t kSpinLimit = 1u << 22;

// ------------------------------------------------------------------ mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// bounded wait for the phase with the given parity; false on timeout
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; i++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kRingConsumerWarps * 32) : "memory");
}

// ------------------------------------------------------------------ plan
// A stage is R consecutive units of the CTA's range with the full K of every row,
// laid out side-major in its ring slot: slot i = side * R + j holds the nibble row
// (K/2 bytes) and, after all nibble rows, the fp16 scale row (K/16 bytes).  Rows of
// one side of a stage are mostly consecutive in HBM, so a stage costs a handful of
// large bulk copies.  Consumer warps form G = 24 / R groups of R/2 warps; group gi
// consumes stages gi, gi+G, ...  When a CTA has more stages than ring slots, the
// ring depth S is a multiple of G so that every use of a slot belongs to the same
// group (each mbarrier phase is then awaited in order by the only warps that
// consume it); otherwise every stage has its own slot and is used once.
struct RingPlan {
  int units;        // total units (pairs or rows)
  int R;            // units per stage (divides 24, even)
  int stages;       // ring depth S (multiple of 24 / R)
  int stage_bytes;  // bytes of one ring slot
  int ring_offset;  // byte offset of the ring in dynamic shared memory
  int bar_offset;   // byte offset of the mbarriers
};

// rows of unit u (pair mode uses the epilogue's pairing; single mode: unit = row)
template <class Epi, int ROWS>
__device__ __forceinline__ void unit_rows(const GemvArgs& g, int u, int& r0, int& r1) {
  if constexpr (ROWS == 2) {
    Epi::rows(g, u, r0, r1);
  } else {
    r0 = u;
    r1 = u;
  }
}

// end of the consumer loop: the argmax epilogue reduces its running key over the
// consumer warps (named barrier: the producer warp has already returned)
template <class Epi>
__device__ __forceinline__ void ring_finish(const GemvArgs& g, EpiState& st, unsigned long long* red) {
  if constexpr (std::is_same<Epi, EpiArgmax>::value) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long k = st.best[0];
#pragma unroll
    for (int off = 16; off >= 1; off /= 2) {
      unsigned long long o = __shfl_xor_sync(0xffffffffu, k, off);
      k = o > k ? o : k;
    }
    if (lane == 0) red[warp] = k;
    consumer_sync();
    if (threadIdx.x == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < kRingConsumerWarps; w++) m = red[w] > m ? red[w] : m;
      if (m) atomicMax(g.argmax_key, m);
    }
  }
}

// NB: blocks per row when known at compile time (0 = runtime, generic loop).
template <class Pro, class Epi, int ROWS, int NB>
__global__ void __launch_bounds__(kRingThreads, 2) q4_gemv_ring_kernel(const GemvArgs g, const RingPlan plan) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  // staged x (xq: 64 B per block, xm: 8 B per block), reduction scratch, norm scratch
  const uint4* xq = reinterpret_cast<const uint4*>(smem_raw);
  const float2* xm = reinterpret_cast<const float2*>(smem_raw + 64 * (g.k >> 5));
  float* red = reinterpret_cast<float*>(smem_raw + 72 * (g.k >> 5));  // 8 floats + 16 u64
  float* slin = red + 40;                                             // norm prologue: k floats
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + plan.bar_offset);
  unsigned char* ring = smem_raw + plan.ring_offset;
  const int S = plan.stages, R = plan.R;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps_per_stage = R >> 1;
  const int G = kRingUnitsPerRound / R;

  // this CTA's units and stages
  const int u0 = (int)((int64_t)blockIdx.x * plan.units / gridDim.x);
  const int u1 = (int)((int64_t)(blockIdx.x + 1) * plan.units / gridDim.x);
  const int nstages = (u1 - u0 + R - 1) / R;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(smem_u32(&bars[s]), 1);                     // full
      mbar_init(smem_u32(&bars[S + s]), warps_per_stage);   // empty
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_launch_dependents();

  const int nb = g.k >> 5;
  const uint32_t nib_row = (uint32_t)g.k >> 1, sc_row = (uint32_t)nb * 2;
  const uint32_t sc_base = (uint32_t)(R * ROWS) * nib_row;

  if (warp == kRingConsumerWarps) {
    // ------------------------------------------------------------ producer
    int issued = 0;
    bool ok = true;
    for (int st = 0; st < nstages; st++) {
      const int slot = st % S, use = st / S;
      if (use > 0 && !mbar_wait(smem_u32(&bars[S + slot]), (use - 1) & 1)) {
        ok = false;
        break;
      }
      const int ua = u0 + st * R, ub = min(u1, ua + R), nr = ub - ua;
      const uint32_t full = smem_u32(&bars[slot]);
      if (lane == 0) mbar_expect_tx(full, (uint32_t)(nr * ROWS) * (nib_row + sc_row));
      __syncwarp();
      // lane i: side i / nr, unit j = i % nr; runs of consecutive rows share one copy
      const int i = lane, nsl = nr * ROWS;
      int side = 0, j = 0, row = -1;
      if (i < nsl) {
        side = i / nr;
        j = i - side * nr;
        int r0, r1;
        unit_rows<Epi, ROWS>(g, ua + j, r0, r1);
        row = side ? r1 : r0;
      }
      const int prev = __shfl_up_sync(0xffffffffu, row, 1);
      const bool start = (i < nsl) && (j == 0 || row != prev + 1);
      const unsigned starts = __ballot_sync(0xffffffffu, start);
      if (start) {
        // run ends at the next start or at the end of this side
        const unsigned later = starts & ~((2u << i) - 1u);
        const int side_end = (side + 1) * nr;
        int end = later ? (__ffs(later) - 1) : nsl;
        if (end > side_end) end = side_end;
        const int len = end - i;
        unsigned char* sbase = ring + (size_t)slot * plan.stage_bytes;
        const int si = side * R + j;
        bulk_g2s(smem_u32(sbase + (size_t)si * nib_row), g.qs + (size_t)row * nib_row, (uint32_t)len * nib_row, full);
        bulk_g2s(smem_u32(sbase + sc_base + (size_t)si * sc_row), g.d + (size_t)row * nb, (uint32_t)len * sc_row, full);
      }
      issued = st + 1;
    }
    if (!ok && lane == 0 && g.error) atomicExch(g.error, 2);
    // copies still in flight must land before the CTA may exit
    for (int st = issued - S > 0 ? issued - S : 0; st < issued; st++)
      if (!mbar_wait(smem_u32(&bars[st % S]), (st / S) & 1) && lane == 0 && g.error) atomicExch(g.error, 3);
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_wait();
  stage_x<Pro, 1>(g, smem_raw, red, slin, threadIdx.x, kRingConsumerWarps * 32);

  const int hl = lane & 15, half = lane >> 4;
  const int gi = warp / warps_per_stage;
  const int j = (warp - gi * warps_per_stage) * 2 + half;  // unit slot within a stage
  EpiState st_epi;
#pragma unroll
  for (int bt = 0; bt < 8; bt++) st_epi.best[bt] = 0ull;
  bool ok = true;

  if (gi < G) {
    for (int st = gi; st < nstages; st += G) {
      const int slot = st % S, use = st / S;
      if (!mbar_wait(smem_u32(&bars[slot]), use & 1)) {
        ok = false;
        break;
      }
      const int ua = u0 + st * R, nr = min(u1, ua + R) - ua;
      const bool active = j < nr;
      const unsigned char* sbase = ring + (size_t)slot * plan.stage_bytes;
      float acc[ROWS];
#pragma unroll
      for (int rr = 0; rr < ROWS; rr++) acc[rr] = 0.0f;
      if (active) {
        const unsigned char* nib[ROWS];
        const uint16_t* scr[ROWS];
#pragma unroll
        for (int rr = 0; rr < ROWS; rr++) {
          nib[rr] = sbase + (size_t)(rr * R + j) * nib_row;
          scr[rr] = reinterpret_cast<const uint16_t*>(sbase + sc_base + (size_t)(rr * R + j) * sc_row);
        }
        if constexpr (NB > 0) {
          constexpr int BPL = (NB + 15) / 16;
#pragma unroll
          for (int i = 0; i < BPL; i++) {
            const int b = hl + 16 * i;
            if ((NB % 16 == 0) || b < NB) {
              const float2 m = xm[b];
#pragma unroll
              for (int rr = 0; rr < ROWS; rr++) {
                const uint4 q = *reinterpret_cast<const uint4*>(nib[rr] + (size_t)b * 16);
                acc[rr] = block_accum(acc[rr], scr[rr][b], q, xq + b, NB, m);
              }
            }
          }
        } else {
#pragma unroll 2
          for (int b = hl; b < nb; b += 16) {
            const float2 m = xm[b];
#pragma unroll
            for (int rr = 0; rr < ROWS; rr++) {
              const uint4 q = *reinterpret_cast<const uint4*>(nib[rr] + (size_t)b * 16);
              acc[rr] = block_accum(acc[rr], scr[rr][b], q, xq + b, nb, m);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars[S + slot]));
#pragma unroll
      for (int rr = 0; rr < ROWS; rr++) acc[rr] = butterfly_sum<16>(acc[rr]);
      if (active && hl == 0) {
        const int u = ua + j;
        int r0, r1;
        unit_rows<Epi, ROWS>(g, u, r0, r1);
        if constexpr (ROWS == 2) {
          Epi::store(g, st_epi, 0, u, r0, r1, acc[0], acc[1]);
        } else {
          Epi::store_row(g, st_epi, 0, r0, acc[0]);
        }
      }
    }
  }
  if (!ok && lane == 0 && g.error) atomicExch(g.error, 4);
  ring_finish<Epi>(g, st_epi, reinterpret_cast<unsigned long long*>(red + 8));
}

}  // namespace spark
