// spark_b200.cu -- C ABI entry points (declared in include/spark_b200.h).
//
// Argument validation happens here, on the host, before any launch: shapes,
// alignment and sizes that the kernels rely on are checked and reported as
// status codes.  Launches use cudaLaunchKernelEx with programmatic stream
// serialization (PDL) so that consecutive kernels of a decode step overlap their
// launch and prologue with the tail of the previous kernel.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <utility>

#include "attention.cuh"
#include "misc.cuh"
#include "q4_gemv.cuh"
#include "q4_gemm_tc.cuh"
#include "q4_gemv_ring.cuh"
#include "spark_b200.h"
#include "step_kernel.cuh"

using namespace spark;

// Device error word: set by kernels whose bounded waits time out (never by a
// successful run).  Read with spark_read_device_error.
__device__ int g_spark_error_word;

namespace {

int g_pdl = 1;
int g_ring = 1;
constexpr int kRingSmemBudget = 227 * 1024;

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// cudaFuncSetAttribute is per (function, device).  Remember which pairs are done so
// that launches during stream capture make no further attribute calls.
struct SmemDone {
  const void* fn;
  int dev;
  size_t bytes;
};
SmemDone g_smem_done[512];
int g_smem_count = 0;
std::mutex g_smem_mu;

int set_smem(const void* kernel, size_t smem) {
  if (smem <= 48 * 1024) return kOk;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrLaunch;
  std::lock_guard<std::mutex> lock(g_smem_mu);
  for (int i = 0; i < g_smem_count; i++)
    if (g_smem_done[i].fn == kernel && g_smem_done[i].dev == dev && g_smem_done[i].bytes >= smem) return kOk;
  // always request the maximum so one call serves every later size
  const int max_bytes = 227 * 1024;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_bytes) != cudaSuccess)
    return kErrLaunch;
  for (int i = 0; i < g_smem_count; i++)
    if (g_smem_done[i].fn == kernel && g_smem_done[i].dev == dev) {
      g_smem_done[i].bytes = max_bytes;
      return kOk;
    }
  if (g_smem_count < 512) g_smem_done[g_smem_count++] = {kernel, dev, (size_t)max_bytes};
  return kOk;
}

template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
  if (set_smem(reinterpret_cast<const void*>(kernel), smem) != kOk) return kErrLaunch;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = g_pdl;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  return e == cudaSuccess ? kOk : kErrLaunch;
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return kNumSMs;
  if (!cached[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : kNumSMs;
  }
  return cached[dev];
}

// ------------------------------------------------------------------ GEMV dispatch
template <class Pro, class Epi, int BATCH>
int gemv_launch_b(const GemvArgs& g, cudaStream_t st) {
  const int nb = g.k / 32;
  const int bpl = (nb + 15) / 16;  // blocks per lane
  const int npairs = g.n / 2;
  const int duos = (npairs + 1) / 2;
  const int sms = num_sms();
  const int ctas_per_sm = 2;
  const int cap = sms * ctas_per_sm;
  int grid = (duos + 7) / 8;  // CTAs of 8 busy warps
  if (grid < sms) grid = duos < sms ? duos : sms;  // spread thin work over all SMs
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  const size_t smem = (size_t)BATCH * (g.k / 32) * 72 + 160 + (Pro::kNorm ? (size_t)g.k * 4 : 0);
  if (smem > 227 * 1024) return kErrTooLarge;
  if (bpl <= 2) return launch(q4_gemv_kernel<Pro, Epi, BATCH, 2>, dim3(grid), dim3(256), smem, st, g);
  if (bpl <= 5) return launch(q4_gemv_kernel<Pro, Epi, BATCH, 5>, dim3(grid), dim3(256), smem, st, g);
  if (bpl <= 8) return launch(q4_gemv_kernel<Pro, Epi, BATCH, 8>, dim3(grid), dim3(256), smem, st, g);
  return launch(q4_gemv_kernel<Pro, Epi, BATCH, 10>, dim3(grid), dim3(256), smem, st, g);
}

int check_q4(const uint8_t* qs, const uint16_t* d, int n, int k) {
  if (!qs || !d) return kErrInvalidArg;
  if (n <= 0 || k <= 0 || (n & 1) || (k % 32)) return kErrUnsupportedShape;
  if (!aligned(qs, 16) || !aligned(d, 2)) return kErrAlignment;
  return kOk;
}

int* device_error_ptr() {
  static int* cached[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_spark_error_word) != cudaSuccess) return nullptr;
    cached[dev] = static_cast<int*>(p);
  }
  return cached[dev];
}

// The ring kernel copies whole rows, so it needs the fp16 scale rows (K/16 bytes)
// to be multiples of 16 bytes (K % 256 == 0) and 16-byte aligned planes; other
// shapes and batch > 1 use the register-direct kernel.
bool ring_ok(const GemvArgs& g) {
  return g_ring && g.batch == 1 && g.k % 256 == 0 && aligned(g.qs, 16) && aligned(g.d, 16);
}

// units per stage: the largest divisor of 24 (even) whose stage fits ~36 KB, and a
// ring depth that is a multiple of the number of warp groups
int ring_plan_budget(RingPlan& p, int units, int rows_per_unit, int k, bool norm, int total_budget) {
  const int row_bytes = k / 2 + k / 16;
  // staged x (72 B per block) + reduction scratch (40 floats) + linear s for the norm (k floats)
  const int xs_bytes = (k / 32) * 72 + 160 + (norm ? k * 4 : 0);
  p.units = units;
  p.bar_offset = (xs_bytes + 15) / 16 * 16;
  const int budget = total_budget - p.bar_offset - 2 * 24 * 8 - 256;
  const int sms = num_sms();
  const int max_units_cta = (units + sms - 1) / sms;
  static const int kR[] = {24, 12, 8, 6, 4, 2};
  for (int R : kR) {
    const int stage = R * rows_per_unit * row_bytes;
    if (stage > 40 * 1024 && R > 2) continue;
    const int G = 24 / R;
    const int max_stages_cta = (max_units_cta + R - 1) / R;
    int S = budget / stage;
    const int cap = G > (8 / G) * G ? G : (8 / G) * G;
    if (S > cap) S = cap;
    // slots are reused only when a CTA has more stages than slots; then every use of
    // a slot must belong to the same consumer group (S % G == 0)
    if (max_stages_cta > S) S = S / G * G;
    else S = max_stages_cta;
    if (S < 1 || (max_stages_cta > S && S < G)) continue;
    p.R = R;
    p.stages = S;
    p.stage_bytes = (stage + 127) / 128 * 128;
    p.ring_offset = (p.bar_offset + 2 * S * 8 + 127) / 128 * 128;
    if ((size_t)p.ring_offset + (size_t)S * p.stage_bytes > (size_t)total_budget) continue;
    return kOk;
  }
  return kErrTooLarge;
}

int ring_plan(RingPlan& p, int units, int rows_per_unit, int k, bool norm) {
  return ring_plan_budget(p, units, rows_per_unit, k, norm, kRingSmemBudget);
}

template <class Pro, class Epi, int ROWS>
int ring_launch(GemvArgs g, cudaStream_t st) {
  RingPlan p;
  const int units = ROWS == 2 ? g.n / 2 : g.n;
  if (ring_plan(p, units, ROWS, g.k, Pro::kNorm) != kOk) return kErrTooLarge;
  const size_t smem = (size_t)p.ring_offset + (size_t)p.stages * p.stage_bytes;
  int grid = num_sms();
  if (grid > units) grid = units;
  g.error = device_error_ptr();
  // compile-time block counts for the synthetic model's K (2560, 4096, 9728)
  switch (g.k) {
    case 2560:
      return launch(q4_gemv_ring_kernel<Pro, Epi, ROWS, 80>, dim3(grid), dim3(kRingThreads), smem, st, g, p);
    case 4096:
      return launch(q4_gemv_ring_kernel<Pro, Epi, ROWS, 128>, dim3(grid), dim3(kRingThreads), smem, st, g, p);
    case 9728:
      return launch(q4_gemv_ring_kernel<Pro, Epi, ROWS, 304>, dim3(grid), dim3(kRingThreads), smem, st, g, p);
    default:
      return launch(q4_gemv_ring_kernel<Pro, Epi, ROWS, 0>, dim3(grid), dim3(kRingThreads), smem, st, g, p);
  }
}

// plain / argmax epilogues: one row per half warp
template <class Pro, class Epi>
int ring_launch_plain(const GemvArgs& g, cudaStream_t st) {
  return ring_launch<Pro, Epi, 1>(g, st);
}

GemvArgs blank_args() {
  GemvArgs g;
  memset(&g, 0, sizeof(g));
  g.batch = 1;
  return g;
}

}  // namespace

extern "C" {

int spark_version(void) { return 100; }

const char* spark_status_string(int status) {
  switch (status) {
    case SPARK_OK: return "ok";
    case SPARK_ERR_INVALID_ARG: return "invalid argument (null pointer or bad value)";
    case SPARK_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
    case SPARK_ERR_ALIGNMENT: return "pointer alignment violated";
    case SPARK_ERR_LAUNCH: return "CUDA launch failed";
    case SPARK_ERR_TOO_LARGE: return "size exceeds the kernel's limit";
    case SPARK_ERR_CUDA: return "CUDA runtime call failed (allocation or IPC)";
    default: return "unknown status";
  }
}

int spark_set_pdl(int enabled) {
  g_pdl = enabled ? 1 : 0;
  return SPARK_OK;
}

int spark_set_gemv_ring(int enabled) {
  g_ring = enabled ? 1 : 0;
  return SPARK_OK;
}

int spark_read_device_error(int* value, int reset) {
  if (!value) return SPARK_ERR_INVALID_ARG;
  if (cudaMemcpyFromSymbol(value, g_spark_error_word, sizeof(int)) != cudaSuccess) return SPARK_ERR_LAUNCH;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_spark_error_word, &zero, sizeof(int)) != cudaSuccess) return SPARK_ERR_LAUNCH;
  }
  return SPARK_OK;
}

int spark_q4_quantize(const float* w, int64_t rows, int64_t k, uint8_t* qs, uint16_t* d, void* stream) {
  if (!w || !qs || !d) return SPARK_ERR_INVALID_ARG;
  if (rows <= 0 || k <= 0 || k % 32) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (!aligned(w, 16) || !aligned(qs, 16) || !aligned(d, 2)) return SPARK_ERR_ALIGNMENT;
  const int64_t nblocks = rows * (k / 32);
  int64_t grid = (nblocks + 255) / 256;
  if (grid > 65535 * 16) grid = 65535 * 16;
  q4_quantize_kernel<<<(unsigned)grid, 256, 0, as_stream(stream)>>>(w, nblocks, qs, d);
  return cudaGetLastError() == cudaSuccess ? SPARK_OK : SPARK_ERR_LAUNCH;
}

int spark_q4_split_gguf(const uint8_t* blocks, int64_t rows, int64_t k, uint8_t* qs, uint16_t* d, void* stream) {
  if (!blocks || !qs || !d) return SPARK_ERR_INVALID_ARG;
  if (rows <= 0 || k <= 0 || k % 32) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (!aligned(qs, 16) || !aligned(d, 2)) return SPARK_ERR_ALIGNMENT;
  const int64_t nblocks = rows * (k / 32);
  int64_t grid = (nblocks + 255) / 256;
  if (grid > 65535 * 16) grid = 65535 * 16;
  q4_split_kernel<<<(unsigned)grid, 256, 0, as_stream(stream)>>>(blocks, nblocks, qs, d);
  return cudaGetLastError() == cudaSuccess ? SPARK_OK : SPARK_ERR_LAUNCH;
}

int spark_q4_dequantize_bf16(const uint8_t* qs, const uint16_t* d, int64_t rows, int64_t k, uint16_t* w,
                             void* stream) {
  if (!qs || !d || !w) return SPARK_ERR_INVALID_ARG;
  if (rows <= 0 || k <= 0 || k % 32) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (!aligned(qs, 16) || !aligned(d, 2) || !aligned(w, 2)) return SPARK_ERR_ALIGNMENT;
  const int64_t nblocks = rows * (k / 32);
  int64_t grid = (nblocks + 255) / 256;
  if (grid > 65535 * 16) grid = 65535 * 16;
  q4_dequant_bf16_kernel<<<(unsigned)grid, 256, 0, as_stream(stream)>>>(qs, d, nblocks, w);
  return cudaGetLastError() == cudaSuccess ? SPARK_OK : SPARK_ERR_LAUNCH;
}

// cuTensorMapEncodeTiled from the driver, through the runtime's entry-point query (no
// link against libcuda)
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D tensor map: `inner` elements per row (row pitch `pitch` bytes), `outer` rows
static bool encode_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t pitch, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw) {
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int spark_q4_gemm_tc(const uint16_t* x, const uint8_t* qs, const uint16_t* d, uint16_t* y, int t, int n, int k,
                     int* error, int64_t wait_ns, void* stream) {
  if (!x || !qs || !d || !y || !error) return SPARK_ERR_INVALID_ARG;
  if (t <= 0 || n <= 0 || k <= 0 || k % tc::kRK) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (!aligned(x, 16) || !aligned(qs, 16) || !aligned(d, 16) || !aligned(y, 2) || !aligned(error, 4))
    return SPARK_ERR_ALIGNMENT;
  if (set_smem(reinterpret_cast<const void*>(&tc::q4_gemm_tc_kernel), tc::kSmemBytes)) return SPARK_ERR_LAUNCH;
  // 256-token tiles for every shape: 128-token tiles dequantize twice the weights per
  // product and measured slower even where they fill the SMs better (o / down: 320
  // tiles of 128 tokens 121 / 272 us, 160 tiles of 256 tokens 88 / 187 us)
  const int sms = num_sms();
  const long long ntm = (n + tc::kBM - 1) / tc::kBM;
  const int bn = tc::kBNMax;
  CUtensorMap mx, mq, md;
  if (!encode_map(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)k, (uint64_t)t, (uint64_t)k * 2, tc::kBK,
                  (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map(&mq, CU_TENSOR_MAP_DATA_TYPE_UINT8, qs, (uint64_t)k / 2, (uint64_t)n, (uint64_t)k / 2,
                  tc::kRK / 2, tc::kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map(&md, CU_TENSOR_MAP_DATA_TYPE_UINT16, d, (uint64_t)k / 32, (uint64_t)n, (uint64_t)k / 16,
                  tc::kRK / 32, tc::kBM, CU_TENSOR_MAP_SWIZZLE_NONE))
    return SPARK_ERR_LAUNCH;
  const long long ntiles = ntm * ((t + bn - 1) / bn);
  const int grid = (int)std::min<long long>(ntiles, sms);
  const unsigned long long limit = wait_ns < 0 ? tc::kWaitNs : (unsigned long long)wait_ns;
  tc::q4_gemm_tc_kernel<<<grid, tc::kThreads, tc::kSmemBytes, as_stream(stream)>>>(mx, mq, md, y, t, n, k, bn,
                                                                                   error, limit);
  return cudaGetLastError() == cudaSuccess ? SPARK_OK : SPARK_ERR_LAUNCH;
}

int spark_q4_gemv(const uint16_t* x, const uint8_t* qs, const uint16_t* d, uint16_t* y, int n, int k, int batch,
                  void* stream) {
  int st = check_q4(qs, d, n, k);
  if (st) return st;
  if (!x || !y) return SPARK_ERR_INVALID_ARG;
  if (batch < 1 || batch > 8) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (!aligned(x, 16) || !aligned(y, 4)) return SPARK_ERR_ALIGNMENT;
  GemvArgs g = blank_args();
  g.qs = qs;
  g.d = d;
  g.n = n;
  g.k = k;
  g.batch = batch;
  g.x = x;
  g.y = y;
  cudaStream_t s = as_stream(stream);
  if (ring_ok(g)) return ring_launch_plain<ProPlain, EpiPlain>(g, s);
  if (batch == 1) return gemv_launch_b<ProPlain, EpiPlain, 1>(g, s);
  if (batch == 2) return gemv_launch_b<ProPlain, EpiPlain, 2>(g, s);
  if (batch <= 4) return gemv_launch_b<ProPlain, EpiPlain, 4>(g, s);
  return gemv_launch_b<ProPlain, EpiPlain, 8>(g, s);
}

static int fill_norm(GemvArgs& g, const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps,
                     uint16_t* res_out, int k) {
  if (!gamma) return SPARK_ERR_INVALID_ARG;
  if (!aligned(gamma, 4) || (a && !aligned(a, 4)) || (b && !aligned(b, 4)) || (res_out && !aligned(res_out, 4)))
    return SPARK_ERR_ALIGNMENT;
  if (!(eps >= 0.0f)) return SPARK_ERR_INVALID_ARG;
  g.a = a;
  g.b = b;
  g.gamma = gamma;
  g.eps = eps;
  g.inv_k = (float)(1.0 / (double)k);
  g.res_out = res_out;
  return SPARK_OK;
}

int spark_rmsnorm_q4_gemv(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps, uint16_t* res_out,
                          const uint8_t* qs, const uint16_t* d, uint16_t* y, int n, int k, void* stream) {
  int st = check_q4(qs, d, n, k);
  if (st) return st;
  if (!a || !y) return SPARK_ERR_INVALID_ARG;
  if (!aligned(y, 4)) return SPARK_ERR_ALIGNMENT;
  GemvArgs g = blank_args();
  if ((st = fill_norm(g, a, b, gamma, eps, res_out, k))) return st;
  g.qs = qs;
  g.d = d;
  g.n = n;
  g.k = k;
  g.y = y;
  if (ring_ok(g)) return ring_launch_plain<ProNorm, EpiPlain>(g, as_stream(stream));
  return gemv_launch_b<ProNorm, EpiPlain, 1>(g, as_stream(stream));
}

int spark_rmsnorm_gate_up_silu(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps,
                               uint16_t* res_out, const uint8_t* qs, const uint16_t* d, uint16_t* mid, int n, int k,
                               void* stream) {
  int st = check_q4(qs, d, n, k);
  if (st) return st;
  if (!a || !mid) return SPARK_ERR_INVALID_ARG;
  GemvArgs g = blank_args();
  if ((st = fill_norm(g, a, b, gamma, eps, res_out, k))) return st;
  g.qs = qs;
  g.d = d;
  g.n = n;
  g.k = k;
  g.y = mid;
  if (ring_ok(g)) return ring_launch<ProNorm, EpiSiluMul, 2>(g, as_stream(stream));
  return gemv_launch_b<ProNorm, EpiSiluMul, 1>(g, as_stream(stream));
}

int spark_qkv_rope_kvstore(const uint16_t* a, const uint16_t* b, const uint16_t* embed, const int32_t* token,
                           const uint16_t* gamma, float eps, uint16_t* res_out, const uint8_t* qs, const uint16_t* d,
                           int k, int nq, int nkv, int head_dim, const uint16_t* cos_sin, const int64_t* pos,
                           const int32_t* block_table, const int64_t* slot_mapping, int block_size,
                           uint16_t* k_cache, uint16_t* v_cache, uint16_t* q_out, void* stream) {
  if (nq <= 0 || nkv <= 0 || head_dim <= 0 || (head_dim & 3) || block_size <= 0) return SPARK_ERR_UNSUPPORTED_SHAPE;
  const int n = (nq + 2 * nkv) * head_dim;
  int st = check_q4(qs, d, n, k);
  if (st) return st;
  if ((!a && !(embed && token)) || !cos_sin || !pos || !k_cache || !v_cache || !q_out) return SPARK_ERR_INVALID_ARG;
  if (!slot_mapping && !block_table) return SPARK_ERR_INVALID_ARG;
  if (!aligned(v_cache, 4) || !aligned(k_cache, 2) || !aligned(q_out, 2) || (embed && !aligned(embed, 4)))
    return SPARK_ERR_ALIGNMENT;
  GemvArgs g = blank_args();
  if ((st = fill_norm(g, a, b, gamma, eps, res_out, k))) return st;
  g.embed = embed;
  g.token = token;
  g.qs = qs;
  g.d = d;
  g.n = n;
  g.k = k;
  g.y = q_out;
  g.nq = nq;
  g.nkv = nkv;
  g.head_dim = head_dim;
  g.block_size = block_size;
  g.cos_sin = cos_sin;
  g.pos64 = pos;
  g.block_table = block_table;
  g.slot_mapping = slot_mapping;
  g.k_cache = k_cache;
  g.v_cache = v_cache;
  if (ring_ok(g)) return ring_launch<ProNorm, EpiRope, 2>(g, as_stream(stream));
  return gemv_launch_b<ProNorm, EpiRope, 1>(g, as_stream(stream));
}

int spark_rmsnorm_q4_head_argmax(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps,
                                 const uint8_t* qs, const uint16_t* d, uint16_t* logits, int n, int k,
                                 unsigned long long* argmax_key, void* stream) {
  int st = check_q4(qs, d, n, k);
  if (st) return st;
  if (!a || !logits || !argmax_key) return SPARK_ERR_INVALID_ARG;
  if (!aligned(logits, 4) || !aligned(argmax_key, 8)) return SPARK_ERR_ALIGNMENT;
  GemvArgs g = blank_args();
  if ((st = fill_norm(g, a, b, gamma, eps, nullptr, k))) return st;
  g.qs = qs;
  g.d = d;
  g.n = n;
  g.k = k;
  g.y = logits;
  g.argmax_key = argmax_key;
  if (ring_ok(g)) return ring_launch_plain<ProNorm, EpiArgmax>(g, as_stream(stream));
  return gemv_launch_b<ProNorm, EpiArgmax, 1>(g, as_stream(stream));
}

static int attn_launch(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                       const int32_t* block_table, const int64_t* pos, const int32_t* seq_len, int nq, int nkv,
                       int head_dim, int block_size, int splits, int max_split_tokens, float scale, float* part_o,
                       float* part_lse, int* error, int* counters, uint16_t* out, void* stream) {
  if (!q || !k_cache || !v_cache || !block_table || !part_o || !part_lse || (!pos && !seq_len))
    return SPARK_ERR_INVALID_ARG;
  if (head_dim != 128 || nkv <= 0 || nq != 4 * nkv || block_size <= 0) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (splits <= 0 || splits > 4096) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (out && (!counters || splits > kAttnMaxFusedSplits)) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (max_split_tokens <= 0 || max_split_tokens > kAttnMaxSplitTokens) return SPARK_ERR_TOO_LARGE;
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(part_o, 16) || !aligned(q, 16))
    return SPARK_ERR_ALIGNMENT;
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  a.q = q;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.block_table = block_table;
  a.pos64 = seq_len ? nullptr : pos;
  a.seq_len32 = seq_len;
  a.nq = nq;
  a.nkv = nkv;
  a.block_size = block_size;
  a.splits = splits;
  a.t_alloc = (max_split_tokens + 15) / 16 * 16;
  const int nch = (a.t_alloc + kAttnChunk - 1) / kAttnChunk;
  a.kv_slots = nch < 2 ? nch : 2;
  a.scale = scale;
  a.part_o = part_o;
  a.part_lse = part_lse;
  a.error = error;
  a.counters = counters;
  a.out = out;
  const int G = 4;
  // the whole split in shared memory, 16 warps (pages of >= 64 tokens: at most 8 page segments)
  if (a.t_alloc <= kWideMaxTokens && block_size >= 64 && (kWideMaxTokens + block_size - 1) / block_size + 1 <= kWideMaxSegs)
    return launch(attn_decode_wide_kernel<128, 4>, dim3(splits, nkv), dim3(kWideThreads),
                  attn_wide_smem(a.t_alloc), as_stream(stream), a);
  const size_t smem = (size_t)(G * a.t_alloc + 2 * G + G * kAttnMaxFusedSplits + 4) * sizeof(float) +
                      (size_t)a.kv_slots * kAttnChunk * (kKRowBytes + kVRowBytes);
  return launch(attn_decode_kernel<128, 4>, dim3(splits, nkv), dim3(kAttnThreads), smem, as_stream(stream), a);
}

int spark_attn_splitkv(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                       const int32_t* block_table, const int64_t* pos, const int32_t* seq_len, int nq, int nkv,
                       int head_dim, int block_size, int splits, int max_split_tokens, float scale, float* part_o,
                       float* part_lse, int* error, void* stream) {
  return attn_launch(q, k_cache, v_cache, block_table, pos, seq_len, nq, nkv, head_dim, block_size, splits,
                     max_split_tokens, scale, part_o, part_lse, error, nullptr, nullptr, stream);
}

int spark_attn_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                      const int32_t* block_table, const int64_t* pos, const int32_t* seq_len, int nq, int nkv,
                      int head_dim, int block_size, int splits, int max_split_tokens, float scale, float* part_o,
                      float* part_lse, int* counters, uint16_t* out, int* error, void* stream) {
  if (!out || !counters) return SPARK_ERR_INVALID_ARG;
  if (!aligned(counters, 4) || !aligned(out, 2)) return SPARK_ERR_ALIGNMENT;
  return attn_launch(q, k_cache, v_cache, block_table, pos, seq_len, nq, nkv, head_dim, block_size, splits,
                     max_split_tokens, scale, part_o, part_lse, error, counters, out, stream);
}

// ------------------------------------------------------------------ allocation-free attention
// Some callers cannot allocate device memory when they decode: a host framework
// that owns every byte of GPU memory and hands out none to plugins, or a real-time
// loop that must never call cudaMalloc after start-up (it can synchronise the device
// and fail under memory pressure).  spark_attn_decode_noalloc gives them the fused
// split-KV attention without any caller-provided workspace: the partial outputs, the
// log-sum-exp values and the per-kv-head arrival counters live in the file-scope
// array below, which every GPU that loads this library keeps until the process exits.
constexpr int kNoAllocMaxSplits = 64;
constexpr int kNoAllocMaxQHeads = 64;
constexpr int kNoAllocMaxKvHeads = 64;
constexpr size_t kNoAllocPartOFloats = (size_t)kNoAllocMaxSplits * kNoAllocMaxQHeads * 128;
constexpr size_t kNoAllocLseFloats = (size_t)kNoAllocMaxSplits * kNoAllocMaxQHeads;
constexpr size_t kNoAllocScratchFloats = kNoAllocPartOFloats + kNoAllocLseFloats + kNoAllocMaxKvHeads;
// 2,113,792 bytes: partials [64 splits][64 q heads][128] fp32, lse [64][64] fp32, 64 int counters
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

namespace {
float* g_noalloc_base[64] = {nullptr};
std::mutex g_noalloc_mu;

// Once per device, with that device current: look up the device address of the
// scratch array (its name is only a host-side stand-in) and zero the counters.
int noalloc_scratch(float** base) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SPARK_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_base[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return SPARK_ERR_LAUNCH;
    float* f = static_cast<float*>(p);
    if (cudaMemset(f + kNoAllocPartOFloats + kNoAllocLseFloats, 0, kNoAllocMaxKvHeads * sizeof(int)) != cudaSuccess)
      return SPARK_ERR_LAUNCH;
    if (cudaDeviceSynchronize() != cudaSuccess) return SPARK_ERR_LAUNCH;
    g_noalloc_base[dev] = f;
  }
  *base = g_noalloc_base[dev];
  return SPARK_OK;
}
}  // namespace

int spark_attn_decode_noalloc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                              const int32_t* block_table, const int64_t* pos, const int32_t* seq_len, int nq,
                              int nkv, int head_dim, int block_size, int splits, int max_split_tokens, float scale,
                              uint16_t* out, int* error, void* stream) {
  if (!out) return SPARK_ERR_INVALID_ARG;
  if (splits > kNoAllocMaxSplits || nq > kNoAllocMaxQHeads || nkv > kNoAllocMaxKvHeads) return SPARK_ERR_TOO_LARGE;
  if (splits <= 0 || nq <= 0 || nkv <= 0) return SPARK_ERR_UNSUPPORTED_SHAPE;
  float* base = nullptr;
  const int st = noalloc_scratch(&base);
  if (st != SPARK_OK) return st;
  float* part_o = base;
  float* part_lse = base + kNoAllocPartOFloats;
  int* counters = reinterpret_cast<int*>(base + kNoAllocPartOFloats + kNoAllocLseFloats);
  return attn_launch(q, k_cache, v_cache, block_table, pos, seq_len, nq, nkv, head_dim, block_size, splits,
                     max_split_tokens, scale, part_o, part_lse, error, counters, out, stream);
}

int spark_attn_combine(const float* part_o, const float* part_lse, int splits, int nq, int head_dim, uint16_t* out,
                       void* stream) {
  if (!part_o || !part_lse || !out) return SPARK_ERR_INVALID_ARG;
  if (splits <= 0 || splits > 4096 || nq <= 0 || head_dim <= 0) return SPARK_ERR_UNSUPPORTED_SHAPE;
  CombineArgs c;
  c.part_o = part_o;
  c.part_lse = part_lse;
  c.splits = splits;
  c.nq = nq;
  c.dim = head_dim;
  c.out = out;
  if (head_dim == 128 && nq % 4 == 0 && splits <= kAttnMaxFusedSplits && aligned(part_o, 16)) {
    const size_t smem = (size_t)(4 * kAttnMaxFusedSplits + 8) * sizeof(float) + 64 * 1024;
    return launch(attn_combine4_kernel, dim3(nq / 4), dim3(128), smem, as_stream(stream), c);
  }
  return launch(attn_combine_kernel, dim3(nq), dim3(128), (size_t)splits * sizeof(float), as_stream(stream), c);
}

int spark_decode_finalize(unsigned long long* argmax_key, int32_t* token_out, int32_t* token_log, int32_t* step,
                          int64_t* pos, void* stream) {
  if (!argmax_key || !token_out) return SPARK_ERR_INVALID_ARG;
  if (token_log && !step) return SPARK_ERR_INVALID_ARG;
  return launch(decode_finalize_kernel, dim3(1), dim3(32), 0, as_stream(stream), argmax_key, token_out, token_log,
                step, pos);
}

int spark_add_rmsnorm(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps, int hidden,
                      uint16_t* res_out, uint16_t* y, void* stream) {
  if (!a || !gamma || !y) return SPARK_ERR_INVALID_ARG;
  if (hidden <= 0 || hidden > 16384) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (!(eps >= 0.0f)) return SPARK_ERR_INVALID_ARG;
  const float inv_h = (float)(1.0 / (double)hidden);
  return launch(add_rmsnorm_kernel, dim3(1), dim3(1024), (size_t)hidden * sizeof(float), as_stream(stream), a, b,
                gamma, eps, inv_h, hidden, res_out, y);
}

int spark_silu_mul(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* out, void* stream) {
  if (!g || !u || !out) return SPARK_ERR_INVALID_ARG;
  if (n <= 0) return SPARK_ERR_UNSUPPORTED_SHAPE;
  int64_t grid = (n + 255) / 256;
  if (grid > 4 * num_sms()) grid = 4 * num_sms();
  return launch(silu_mul_kernel, dim3((unsigned)grid), dim3(256), 0, as_stream(stream), g, u, n, out);
}

int spark_add_rmsnorm_rows(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps, int rows,
                           int hidden, uint16_t* res_out, uint16_t* y, void* stream) {
  if (!a || !gamma || !y) return SPARK_ERR_INVALID_ARG;
  if (rows <= 0 || hidden <= 0 || hidden > 12288) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (hidden % 8 == 0 && hidden <= 256 * 8 * kRowGroupsPerThread && aligned(a, 16) && (!b || aligned(b, 16)) &&
      aligned(gamma, 16) && aligned(y, 16) && (!res_out || aligned(res_out, 16)))
    return launch(add_rmsnorm_rows_v8_kernel, dim3((unsigned)rows), dim3(256), 0, as_stream(stream), a, b, gamma,
                  eps, (float)(1.0 / (double)hidden), hidden, res_out, y);
  return launch(add_rmsnorm_rows_kernel, dim3((unsigned)rows), dim3(256), (size_t)(hidden + 8) * sizeof(float),
                as_stream(stream), a, b, gamma, eps, (float)(1.0 / (double)hidden), hidden, res_out, y);
}

int spark_rope_neox_rows(uint16_t* x, int64_t row_stride, int rows, int nh, int head_dim, int rotary_dim,
                         const uint16_t* cos_sin, int64_t pos0, void* stream) {
  if (!x || !cos_sin) return SPARK_ERR_INVALID_ARG;
  if (rows <= 0 || nh <= 0 || head_dim <= 0 || rotary_dim <= 0 || rotary_dim > head_dim || rotary_dim % 2 ||
      pos0 < 0 || row_stride < (int64_t)nh * head_dim)
    return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (rotary_dim % 16 == 0 && head_dim % 8 == 0 && row_stride % 8 == 0 && aligned(x, 16) && aligned(cos_sin, 16)) {
    const int64_t total8 = (int64_t)rows * nh * (rotary_dim / 16);
    const int64_t grid8 = std::min<int64_t>((total8 + 255) / 256, 16LL * num_sms());
    return launch(rope_rows_v8_kernel, dim3((unsigned)grid8), dim3(256), 0, as_stream(stream), x, row_stride, rows,
                  nh, head_dim, rotary_dim, cos_sin, pos0);
  }
  const int64_t total = (int64_t)rows * nh * (rotary_dim / 2);
  const int64_t grid = std::min<int64_t>((total + 255) / 256, 16LL * num_sms());
  return launch(rope_rows_kernel, dim3((unsigned)grid), dim3(256), 0, as_stream(stream), x, row_stride, rows, nh,
                head_dim, rotary_dim, cos_sin, pos0);
}

int spark_act_mul_rows(const uint16_t* gu, int rows, int inter, const uint16_t* gelu_table, uint16_t* out,
                       void* stream) {
  if (!gu || !out) return SPARK_ERR_INVALID_ARG;
  if (rows <= 0 || inter <= 0) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (inter % 8 == 0 && rows <= 65535 && aligned(gu, 16) && aligned(out, 16))
    return launch(act_mul_rows_v8_kernel, dim3((unsigned)((inter / 8 + 255) / 256), (unsigned)rows), dim3(256), 0,
                  as_stream(stream), gu, inter, gelu_table, out);
  const int64_t total = (int64_t)rows * inter;
  const int64_t grid = std::min<int64_t>((total + 255) / 256, 16LL * num_sms());
  return launch(act_mul_rows_kernel, dim3((unsigned)grid), dim3(256), 0, as_stream(stream), gu, (int64_t)rows,
                inter, gelu_table, out);
}

int spark_rope_neox(uint16_t* x, int nh, int head_dim, const uint16_t* cos_sin, const int64_t* pos, void* stream) {
  if (!x || !cos_sin || !pos) return SPARK_ERR_INVALID_ARG;
  if (nh <= 0 || head_dim <= 0 || (head_dim & 1)) return SPARK_ERR_UNSUPPORTED_SHAPE;
  const int total = nh * head_dim / 2;
  const int grid = (total + 255) / 256;
  return launch(rope_neox_kernel, dim3(grid), dim3(256), 0, as_stream(stream), x, nh, head_dim, cos_sin, pos);
}

int spark_slot_mapping(int64_t num_tokens, int64_t max_tokens, const int32_t* query_start, const int64_t* positions,
                       const int32_t* block_table, int64_t block_size, int64_t* out, void* stream) {
  if (!query_start || !out || (num_tokens > 0 && (!positions || !block_table))) return SPARK_ERR_INVALID_ARG;
  if (num_tokens < 0 || max_tokens <= 0 || num_tokens > max_tokens || block_size <= 0)
    return SPARK_ERR_UNSUPPORTED_SHAPE;
  int64_t grid = (max_tokens + 255) / 256;
  if (grid > 4 * num_sms()) grid = 4 * num_sms();
  return launch(slot_mapping_kernel, dim3((unsigned)grid), dim3(256), 0, as_stream(stream), num_tokens, max_tokens,
                query_start, positions, block_table, block_size, out);
}

int spark_kv_store(const uint16_t* k, const uint16_t* v, const int64_t* slot_mapping, int64_t tokens, int nkv,
                   int head_dim, int block_size, uint16_t* k_cache, uint16_t* v_cache, void* stream) {
  if (!k || !v || !slot_mapping || !k_cache || !v_cache) return SPARK_ERR_INVALID_ARG;
  if (tokens < 0 || nkv <= 0 || head_dim <= 0 || head_dim % 8 || block_size <= 0) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(k_cache) |
       reinterpret_cast<uintptr_t>(v_cache)) & 15)
    return SPARK_ERR_ALIGNMENT;
  if (tokens == 0) return SPARK_OK;
  const int64_t total = tokens * nkv * head_dim / 8 * 2;
  int64_t grid = (total + 255) / 256;
  if (grid > 4 * num_sms()) grid = 4 * num_sms();
  return launch(kv_store_kernel, dim3((unsigned)grid), dim3(256), 0, as_stream(stream), k, v, slot_mapping, tokens,
                nkv, head_dim, (int64_t)block_size, k_cache, v_cache);
}

// ------------------------------------------------------------------ persistent decode step
int64_t spark_t16_bytes(int n, int k, int kp) {
  if (n <= 0 || k <= 0 || kp <= 0 || k % kp) return -1;
  return (int64_t)(n / 16) * kp * 9 * (k / kp);
}

int spark_q4_pack_t16(const uint8_t* qs, const uint16_t* d, int n, int k, int kp, int rowmap, int aux, uint8_t* out,
                      void* stream) {
  if (!qs || !d || !out) return SPARK_ERR_INVALID_ARG;
  if (n <= 0 || k <= 0 || kp <= 0 || n % 16 || k % kp || (k / kp) % 64) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (rowmap == SPARK_ROWS_PAIR_HALF) {  // aux = head_dim | rotary_dim << 16
    const int hd = aux & 0xffff, rot = (aux >> 16) & 0xffff;
    if (aux < 0 || hd <= 0 || hd % 16 || (n % hd) % 16 || rot % 16 || rot > hd) return SPARK_ERR_UNSUPPORTED_SHAPE;
  } else if (rowmap == SPARK_ROWS_GATE_UP) {
    if ((n / 2) % 8) return SPARK_ERR_UNSUPPORTED_SHAPE;
  } else if (rowmap != SPARK_ROWS_PLAIN) {
    return SPARK_ERR_INVALID_ARG;
  }
  if ((reinterpret_cast<uintptr_t>(qs) | reinterpret_cast<uintptr_t>(out)) & 15) return SPARK_ERR_ALIGNMENT;
  if (reinterpret_cast<uintptr_t>(d) & 3) return SPARK_ERR_ALIGNMENT;
  const int64_t total = (int64_t)(n / 16) * kp * ((k / kp) / 64) * 32;
  int64_t grid = (total + 255) / 256;
  if (grid > 16 * num_sms()) grid = 16 * num_sms();
  return launch(step::t16_pack_kernel, dim3((unsigned)grid), dim3(256), 0, as_stream(stream), qs, d, n, k, kp, rowmap,
                aux, out);
}

int64_t spark_t6_bytes(int n, int k) { return (int64_t)n * k * 105 / 128; }

int spark_q6k_pack_t6(const uint8_t* blocks, int n, int k, int kp, uint8_t* out, void* stream) {
  if (!blocks || !out) return SPARK_ERR_INVALID_ARG;
  if (n <= 0 || k <= 0 || kp <= 0 || n % 16 || k % 256 || k % kp || (k / kp) % 256) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (reinterpret_cast<uintptr_t>(out) & 15) return SPARK_ERR_ALIGNMENT;
  const int64_t total = (int64_t)(n / 16) * kp * ((k / kp) / 64) * 32;
  int64_t grid = (total + 255) / 256;
  if (grid > 16 * num_sms()) grid = 16 * num_sms();
  step::t6_pack_kernel<<<(unsigned)grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(blocks, n, k, kp, out);
  return cudaGetLastError() == cudaSuccess ? SPARK_OK : SPARK_ERR_LAUNCH;
}

int spark_q6k_dequantize(const uint8_t* blocks, int64_t nblocks, float* out, void* stream) {
  if (!blocks || !out || nblocks < 0) return SPARK_ERR_INVALID_ARG;
  if (nblocks == 0) return SPARK_OK;
  int64_t grid = (nblocks * 256 + 255) / 256;
  if (grid > 16 * num_sms()) grid = 16 * num_sms();
  step::q6k_dequant_kernel<<<(unsigned)grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(blocks, nblocks, out);
  return cudaGetLastError() == cudaSuccess ? SPARK_OK : SPARK_ERR_LAUNCH;
}

int spark_step_ring_bytes(void) { return step::kRingBytes; }

int spark_step_ring_bytes_batch(int batch) {
  switch (batch) {
    case 1: return step::Layout<1>::ring;
    case 2: return step::Layout<2>::ring;
    case 4: return step::Layout<4>::ring;
    case 8: return step::Layout<8>::ring;
    default: return 0;
  }
}

static int batch_scratch(int nb) {
  return nb == 2 ? step::Layout<2>::scratch : nb == 4 ? step::Layout<4>::scratch : step::Layout<8>::scratch;
}

// a stage of a batch program (batch 2, 4 or 8): the subset of the stage forms the batch
// kernels carry, and the shared-memory sizes of NB staged inputs
static int check_batch_stage(const SparkStage& s, int ncta) {
  const int nb = s.batch;
  if (nb != 2 && nb != 4 && nb != 8) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (s.xchg || s.gate || s.window || s.table) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (s.kind == SPARK_STAGE_ATTN) {
    if (s.head_dim != 128 || s.bt_stride <= 0) return SPARK_ERR_UNSUPPORTED_SHAPE;
    return SPARK_OK;
  }
  if (s.kind != SPARK_STAGE_GEMV) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (s.pro != SPARK_PRO_BF16 && (s.pro != SPARK_PRO_PARTS || !s.norm)) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (s.epi == SPARK_EPI_GELU_MUL || s.ks > 2) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (s.epi == SPARK_EPI_ROPE_KV &&
      (s.head_dim != 128 || (s.rotary_dim && s.rotary_dim != 128) || s.bt_stride <= 0))
    return SPARK_ERR_UNSUPPORTED_SHAPE;
  const int ring = spark_step_ring_bytes_batch(nb), scratch = batch_scratch(nb);
  if (9 * (s.k / s.kp) > ring) return SPARK_ERR_TOO_LARGE;
  if (s.norm) {  // fp32 pre-norm vectors + gamma; items per thread
    if ((int64_t)4 * s.k * nb + 2 * s.k > scratch) return SPARK_ERR_TOO_LARGE;
    if ((int64_t)nb * (s.k / 8) > (int64_t)step::kBatchItems * step::kConsumers) return SPARK_ERR_TOO_LARGE;
  } else {
    const bool part_x = s.kp > 1 && ncta % s.kp == 0;
    const int kx = part_x ? s.k / s.kp : s.k;
    if ((int64_t)72 * (kx / 32) * nb > scratch) return SPARK_ERR_TOO_LARGE;
  }
  return SPARK_OK;
}

int spark_step_num_ctas(void) { return num_sms(); }

static int check_stage(const SparkStage& s, int i, int ncta) {
  if (s.wait >= i || s.wait < -1) return SPARK_ERR_INVALID_ARG;
  if (s.batch < 0 || s.bt_stride < 0) return SPARK_ERR_INVALID_ARG;
  if (s.kind == SPARK_STAGE_GEMV_Q6) {  // Q6_K weights: plain rows, whole super-blocks per part
    if (s.k <= 0 || s.kp <= 0 || s.k % s.kp || (s.k / s.kp) % 256 || s.rowmap != SPARK_ROWS_PLAIN)
      return SPARK_ERR_UNSUPPORTED_SHAPE;
    if (s.ks <= 0 || ((s.k / s.kp) / 32) % s.ks) return SPARK_ERR_UNSUPPORTED_SHAPE;
    if (step::t6_unit_bytes(s.k / s.kp) > (uint32_t)step::kRingBytes) return SPARK_ERR_TOO_LARGE;
    if (72 * (s.k / 32) + 6 * s.k + 8 * (s.k / 32) > step::kScratchBytes) return SPARK_ERR_TOO_LARGE;
    if (s.epi != SPARK_EPI_BF16 && s.epi != SPARK_EPI_PARTS && s.epi != SPARK_EPI_ARGMAX) return SPARK_ERR_INVALID_ARG;
  }
  if (s.kind == SPARK_STAGE_GEMV || s.kind == SPARK_STAGE_GEMV_Q6) {
    if (!s.w || (!s.a && !s.embed && s.pro != SPARK_PRO_ATTN)) return SPARK_ERR_INVALID_ARG;
    if (s.n <= 0 || s.n % 16 || s.k <= 0 || s.kp <= 0 || s.k % s.kp || (s.k / s.kp) % 64 || s.ks <= 0 ||
        (s.kind == SPARK_STAGE_GEMV && ((s.k / s.kp) / 64) % s.ks))
      return SPARK_ERR_UNSUPPORTED_SHAPE;
    if (s.units != s.n / 16 * s.kp || s.rot < 0 || s.rot >= ncta) return SPARK_ERR_INVALID_ARG;
    if (s.row0 < 0 || (s.row0 && s.epi != SPARK_EPI_ARGMAX) || s.xchg < 0 || s.xchg > SPARK_XCHG_TAGGED)
      return SPARK_ERR_INVALID_ARG;
    if (s.xchg == SPARK_XCHG_TAGGED && s.epi != SPARK_EPI_PARTS) return SPARK_ERR_INVALID_ARG;
    if (s.pro == SPARK_PRO_PARTS_TAGGED && (reinterpret_cast<uintptr_t>(s.a) & 15)) return SPARK_ERR_ALIGNMENT;
    if (s.batch <= 1) {  // (batch programs: check_batch_stage)
      if (s.kind == SPARK_STAGE_GEMV && 9 * (s.k / s.kp) > step::kRingBytes) return SPARK_ERR_TOO_LARGE;
      if (72 * (s.k / 32) + (s.norm ? 6 * s.k : 0) > step::kScratchBytes) return SPARK_ERR_TOO_LARGE;
    }
    if (s.ks > step::kMaxSlices) return SPARK_ERR_UNSUPPORTED_SHAPE;
    if (s.norm && (reinterpret_cast<uintptr_t>(s.gamma) & 15)) return SPARK_ERR_ALIGNMENT;
    if (s.batch <= 1 && s.k > step::kStageGroups * step::kConsumers * 8) return SPARK_ERR_TOO_LARGE;
    if ((reinterpret_cast<uintptr_t>(s.a) | reinterpret_cast<uintptr_t>(s.b) | reinterpret_cast<uintptr_t>(s.embed) |
         reinterpret_cast<uintptr_t>(s.gamma) | reinterpret_cast<uintptr_t>(s.res_out)) & 15)
      return SPARK_ERR_ALIGNMENT;
    if (s.pro == SPARK_PRO_PARTS || s.pro == SPARK_PRO_PARTS_TAGGED) {
      if (s.a_parts <= 0 || s.a_parts > step::kMaxParts || !s.a || s.embed) return SPARK_ERR_INVALID_ARG;
      if (s.batch <= 1 && s.k > step::kConsumers * 8) return SPARK_ERR_TOO_LARGE;  // one 8-element group per thread
    } else if (s.pro == SPARK_PRO_ATTN) {
      if (s.kind != SPARK_STAGE_GEMV || s.norm || s.embed || s.wait != -1) return SPARK_ERR_INVALID_ARG;
      if (s.splits <= 0 || (int64_t)s.kp * s.splits > ncta) return SPARK_ERR_INVALID_ARG;
    } else if (s.pro != SPARK_PRO_BF16) {
      return SPARK_ERR_INVALID_ARG;
    }
    if (s.embed && !s.token) return SPARK_ERR_INVALID_ARG;
    if (s.norm && !s.gamma) return SPARK_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(s.w) & 15) return SPARK_ERR_ALIGNMENT;
    switch (s.epi) {
      case SPARK_EPI_BF16:
        if (s.kp != 1 || !s.out) return SPARK_ERR_INVALID_ARG;
        break;
      case SPARK_EPI_PARTS:
        if (!s.out) return SPARK_ERR_INVALID_ARG;
        break;
      case SPARK_EPI_SILU_MUL:
        if (s.kp != 1 || !s.out || s.rowmap != SPARK_ROWS_GATE_UP) return SPARK_ERR_INVALID_ARG;
        break;
      case SPARK_EPI_GELU_MUL:
        if (s.kp != 1 || !s.out || !s.table || s.rowmap != SPARK_ROWS_GATE_UP) return SPARK_ERR_INVALID_ARG;
        if (reinterpret_cast<uintptr_t>(s.table) & 1) return SPARK_ERR_ALIGNMENT;
        break;
      case SPARK_EPI_ARGMAX:
        if (s.kp != 1 || !s.key) return SPARK_ERR_INVALID_ARG;
        break;
      case SPARK_EPI_ROPE_KV:
        if (s.kp != 1 || s.rowmap != SPARK_ROWS_PAIR_HALF || !s.q || !s.k_cache || !s.v_cache || !s.kv_new ||
            !s.cos_sin || !s.pos || !s.block_table || s.block_size <= 0 || s.nq <= 0 || s.nkv <= 0)
          return SPARK_ERR_INVALID_ARG;
        if (s.head_dim > 256 || s.head_dim % 16) return SPARK_ERR_UNSUPPORTED_SHAPE;
        if (s.rotary_dim < 0 || s.rotary_dim > s.head_dim || s.rotary_dim % 16) return SPARK_ERR_UNSUPPORTED_SHAPE;
        {  // gate rows (Spark): the heads' gate logits after the q / k / v heads, 16-row padded
          const int gate_rows = s.gate ? (s.nq + 15) / 16 * 16 : 0;
          if (gate_rows >= s.head_dim || s.n != (s.nq + 2 * s.nkv) * s.head_dim + gate_rows)
            return SPARK_ERR_UNSUPPORTED_SHAPE;
        }
        if (reinterpret_cast<uintptr_t>(s.gate) & 1) return SPARK_ERR_ALIGNMENT;
        break;
      default:
        return SPARK_ERR_INVALID_ARG;
    }
    if (s.rowmap == SPARK_ROWS_PAIR_HALF) {
      if (s.head_dim <= 0 || s.head_dim % 16 || (s.n % s.head_dim) % 16) return SPARK_ERR_UNSUPPORTED_SHAPE;
    } else if (s.rowmap != SPARK_ROWS_PLAIN && s.rowmap != SPARK_ROWS_GATE_UP) {
      return SPARK_ERR_INVALID_ARG;
    }
    return SPARK_OK;
  }
  if (s.kind != SPARK_STAGE_ATTN) return SPARK_ERR_INVALID_ARG;
  if (!s.q || !s.k_cache || !s.v_cache || !s.kv_new || !s.pos || !s.block_table || !s.part_o || !s.part_lse ||
      !s.head_counters || !s.attn_out)
    return SPARK_ERR_INVALID_ARG;
  if ((s.head_dim != 128 && s.head_dim != 256) || s.nkv <= 0 || s.nq != 4 * s.nkv || s.block_size <= 0 ||
      s.block_size % step::kRunTokens)
    return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (s.window < 0) return SPARK_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(s.gate) & 1) return SPARK_ERR_ALIGNMENT;
  // (kv head, split) tasks round-robin; the combine keeps 2 x 4 x splits floats in the scratch
  if (s.splits <= 0 || s.splits > step::kMaxCombineSplits) return SPARK_ERR_UNSUPPORTED_SHAPE;
  if (s.max_split_tokens <= 0 || s.max_split_tokens > step::kMaxSplitTokens) return SPARK_ERR_TOO_LARGE;
  if ((reinterpret_cast<uintptr_t>(s.kv_new) | reinterpret_cast<uintptr_t>(s.k_cache) |
       reinterpret_cast<uintptr_t>(s.v_cache) | reinterpret_cast<uintptr_t>(s.part_o) |
       reinterpret_cast<uintptr_t>(s.q)) & 15)
    return SPARK_ERR_ALIGNMENT;
  return SPARK_OK;
}

int spark_window_alloc(unsigned long long bytes, void** ptr) {
  if (!ptr || bytes == 0) return SPARK_ERR_INVALID_ARG;
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return SPARK_ERR_CUDA;
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return SPARK_ERR_CUDA;
  }
  return SPARK_OK;
}

int spark_window_free(void* ptr) { return ptr && cudaFree(ptr) != cudaSuccess ? SPARK_ERR_CUDA : SPARK_OK; }

int spark_ipc_handle(const void* window, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == SPARK_IPC_HANDLE_BYTES, "IPC handle size");
  if (!window || !handle) return SPARK_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(window)) != cudaSuccess) return SPARK_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return SPARK_OK;
}

int spark_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return SPARK_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? SPARK_OK : SPARK_ERR_CUDA;
}

int spark_ipc_close(void* ptr) {
  if (!ptr) return SPARK_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? SPARK_OK : SPARK_ERR_CUDA;
}

static bool in_window(const SparkStepIO& io, const void* p, unsigned long long bytes) {
  const uintptr_t b = reinterpret_cast<uintptr_t>(io.window), a = reinterpret_cast<uintptr_t>(p);
  return p && a >= b && a + bytes <= b + io.window_bytes;
}

// tensor-parallel wiring: exchange stages need the window, and what peers write into
// (counters, parts, key) must lie inside it
static int check_tp(const SparkStage* st, int num_stages, const SparkStepIO& io) {
  bool any = false;
  for (int i = 0; i < num_stages; i++) any = any || st[i].xchg;
  if (io.tp_size <= 1) return any ? SPARK_ERR_INVALID_ARG : SPARK_OK;
  if (io.tp_size > 64 || io.tp_rank < 0 || io.tp_rank >= io.tp_size || !io.peer_windows || !io.window)
    return SPARK_ERR_INVALID_ARG;
  if (!in_window(io, io.counters, sizeof(int32_t) * (num_stages + 3))) return SPARK_ERR_INVALID_ARG;
  for (int i = 0; i < num_stages; i++) {
    const SparkStage& s = st[i];
    if (!s.xchg) continue;
    if (s.kind != SPARK_STAGE_GEMV && s.kind != SPARK_STAGE_GEMV_Q6) return SPARK_ERR_INVALID_ARG;
    if (s.epi == SPARK_EPI_PARTS) {
      const unsigned long long word = s.xchg == SPARK_XCHG_TAGGED ? 8ull : 4ull;
      if (!in_window(io, s.out, word * s.n * s.kp * io.tp_size)) return SPARK_ERR_INVALID_ARG;
    } else if (s.epi == SPARK_EPI_ARGMAX) {
      if (!in_window(io, s.key, 8) || (io.key && io.key != s.key)) return SPARK_ERR_INVALID_ARG;
    } else {
      return SPARK_ERR_INVALID_ARG;
    }
  }
  return SPARK_OK;
}

int spark_step_run(const SparkStage* host_stages, const SparkStage* dev_stages, int num_stages, const SparkStepIO* io,
                   void* stream) {
  if (!host_stages || !io || !io->counters || num_stages <= 0) return SPARK_ERR_INVALID_ARG;
  {
    const int t = check_tp(host_stages, num_stages, *io);
    if (t != SPARK_OK) return t;
  }
  if (num_stages > 1 && !dev_stages) return SPARK_ERR_INVALID_ARG;
  if (dev_stages && (reinterpret_cast<uintptr_t>(dev_stages) & 15)) return SPARK_ERR_ALIGNMENT;
  const int ncta = num_sms();
  for (int i = 0; i < num_stages; i++) {
    const int st = check_stage(host_stages[i], i, ncta);
    if (st != SPARK_OK) return st;
  }
  // batch: one B for the whole program, not tensor parallel, the batch kernels' stage forms
  const int nb = host_stages[0].batch > 1 ? host_stages[0].batch : 1;
  for (int i = 0; i < num_stages; i++) {
    if ((host_stages[i].batch > 1 ? host_stages[i].batch : 1) != nb) return SPARK_ERR_INVALID_ARG;
    if (nb > 1) {
      if (io->tp_size > 1 || host_stages[i].pro == SPARK_PRO_ATTN) return SPARK_ERR_UNSUPPORTED_SHAPE;
      const int st = check_batch_stage(host_stages[i], ncta);
      if (st != SPARK_OK) return st;
    }
  }
  for (int i = 0; i < num_stages; i++)  // a tagged exchange stage is not counted: nothing may wait on it
    if (host_stages[i].xchg == SPARK_XCHG_TAGGED)
      for (int j = i + 1; j < num_stages; j++)
        if (host_stages[j].wait == i) return SPARK_ERR_INVALID_ARG;
  for (int i = 0; i < num_stages; i++) {  // an o_proj fused behind attention: wiring of the pair
    const SparkStage& o = host_stages[i];
    if (o.kind == SPARK_STAGE_ATTN) continue;
    if (o.pro != SPARK_PRO_ATTN) continue;
    if (i == 0) return SPARK_ERR_INVALID_ARG;
    const SparkStage& a = host_stages[i - 1];
    if (a.kind != SPARK_STAGE_ATTN || o.kp != a.nkv || o.k != a.nq * a.head_dim || o.splits != a.splits ||
        o.epi != SPARK_EPI_PARTS)
      return SPARK_ERR_INVALID_ARG;
    for (int j = i; j < num_stages; j++)
      if (host_stages[j].wait == i - 1) return SPARK_ERR_INVALID_ARG;  // nothing waits on the fused attention
  }
  step::StepParams P;
  memset(&P, 0, sizeof(P));
  P.stages = num_stages > 1 ? dev_stages : nullptr;
  P.inline_stage = host_stages[0];
  P.num_stages = num_stages;
  P.io = *io;
  if (!P.io.error) P.io.error = device_error_ptr();
  // Q6_K stages, and attention stages with more (kv head, split) tasks than CTAs, run in
  // the kernel instantiations that have their code
  bool q6 = false, multi = false, spark = false;
  for (int i = 0; i < num_stages; i++) {
    const SparkStage& h = host_stages[i];
    q6 = q6 || h.kind == SPARK_STAGE_GEMV_Q6;
    multi = multi || (h.kind == SPARK_STAGE_ATTN && (int64_t)h.nkv * h.splits > ncta);
    if (h.kind == SPARK_STAGE_ATTN)
      spark = spark || h.head_dim != 128 || h.window > 0 || h.gate;
    else
      spark = spark || h.epi == SPARK_EPI_GELU_MUL ||
              (h.epi == SPARK_EPI_ROPE_KV && (h.gate || (h.rotary_dim && h.rotary_dim != h.head_dim)));
  }
  // the Spark instantiation's attention is head_dim 256, the others' 128
  for (int i = 0; i < num_stages; i++)
    if (host_stages[i].kind == SPARK_STAGE_ATTN && host_stages[i].head_dim != (spark ? 256 : 128))
      return SPARK_ERR_UNSUPPORTED_SHAPE;
  using Kernel = void (*)(const step::StepParams);
  // tensor-parallel programs (tagged exchange reads) run in their own instantiations
  static const Kernel kernels[16] = {
      step::step_kernel<false, false, false, false>, step::step_kernel<false, false, true, false>,
      step::step_kernel<false, true, false, false>,  step::step_kernel<false, true, true, false>,
      step::step_kernel<true, false, false, false>,  step::step_kernel<true, false, true, false>,
      step::step_kernel<true, true, false, false>,   step::step_kernel<true, true, true, false>,
      step::step_kernel<false, false, false, true>,  step::step_kernel<false, false, true, true>,
      step::step_kernel<false, true, false, true>,   step::step_kernel<false, true, true, true>,
      step::step_kernel<true, false, false, true>,   step::step_kernel<true, false, true, true>,
      step::step_kernel<true, true, false, true>,    step::step_kernel<true, true, true, true>};
  // batch programs: one instantiation per B (any number of attention tasks)
  static const Kernel batch_kernels[3] = {step::step_kernel<false, true, false, false, 2>,
                                          step::step_kernel<false, true, false, false, 4>,
                                          step::step_kernel<false, true, false, false, 8>};
  const bool tp = io->tp_size > 1;
  const Kernel kernel =
      nb > 1 ? batch_kernels[nb == 2 ? 0 : (nb == 4 ? 1 : 2)] : kernels[8 * tp + 4 * q6 + 2 * multi + spark];
  if (set_smem(reinterpret_cast<const void*>(kernel), step::kSmemBytes) != kOk) return kErrLaunch;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ncta);
  cfg.blockDim = dim3(step::kThreads);
  cfg.dynamicSmemBytes = step::kSmemBytes;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, P);
  return e == cudaSuccess ? SPARK_OK : SPARK_ERR_LAUNCH;
}

}  // extern "C"
