// Status plumbing, path metadata and the small device-wide primitives
// (exclusive scan, per-row sort) shared by the graph and neighbour-list code.
#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>
#include <cstdarg>
#include <cstdio>

#include "tc_gemm.cuh"

namespace bm {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<long long> g_launches{0};

// ---- launch profiler: an event after every launch on the profiled stream
struct ProfRec {
  const char* name;  // nullptr for a mark
  cudaEvent_t ev;
};
static std::mutex g_prof_mu;
static bool g_prof_on = false;
static cudaStream_t g_prof_stream = nullptr;
static std::vector<ProfRec> g_prof_recs;
static std::vector<cudaEvent_t> g_prof_pool;
struct ProfTotal {
  std::string name;
  long long count;
  double ms;
};
static std::vector<ProfTotal> g_prof_totals;

static void prof_record(const char* name) {
  cudaEvent_t ev;
  if (!g_prof_pool.empty()) {
    ev = g_prof_pool.back();
    g_prof_pool.pop_back();
  } else if (cudaEventCreate(&ev) != cudaSuccess) {
    return;
  }
  cudaEventRecord(ev, g_prof_stream);
  g_prof_recs.push_back({name, ev});
}

int check_launch(const char* what, int launches) {
  g_launches.fetch_add(launches, std::memory_order_relaxed);
  if (g_prof_on && launches > 0) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    prof_record(what);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(BM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return BM_OK;
}

// ------------------------------------------------------------------ scan --
// Phase 1: per-block sums of 1024-element tiles.  Phase 2: one block scans
// the tile sums (looping if there are more than 1024 tiles).  Phase 3: each
// tile scans itself and adds its tile offset.  Integer adds: deterministic.
constexpr int kScanTile = 1024;

__device__ __forceinline__ int64_t block_incl_scan(int64_t v, int64_t* sh) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int64_t u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    int64_t s = (lane < (int)(blockDim.x >> 5)) ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int64_t u = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += u;
    }
    sh[lane] = s;
  }
  __syncthreads();
  if (w > 0) v += sh[w - 1];
  __syncthreads();
  return v;
}

__global__ void scan_tile_sums(const int* __restrict__ in, int64_t n, int64_t* __restrict__ sums) {
  __shared__ int64_t sh[32];
  int64_t i = (int64_t)blockIdx.x * kScanTile + threadIdx.x;
  int64_t v = (i < n) ? in[i] : 0;
  v = block_incl_scan(v, sh);
  if (threadIdx.x == kScanTile - 1) sums[blockIdx.x] = v;
}

__global__ void scan_sums_serial(int64_t* __restrict__ sums, int64_t tiles) {
  __shared__ int64_t sh[32];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < tiles; base += kScanTile) {
    int64_t i = base + threadIdx.x;
    int64_t v = (i < tiles) ? sums[i] : 0;
    int64_t inc = block_incl_scan(v, sh);
    int64_t c = carry;
    if (i < tiles) sums[i] = c + inc - v;  // exclusive tile offset
    __syncthreads();
    if (threadIdx.x == kScanTile - 1) carry = c + inc;
    __syncthreads();
  }
  if (threadIdx.x == 0) sums[tiles] = carry;
}

__global__ void scan_apply(const int* __restrict__ in, int64_t n, const int64_t* __restrict__ sums,
                           int64_t tiles, int64_t* __restrict__ out) {
  __shared__ int64_t sh[32];
  int64_t i = (int64_t)blockIdx.x * kScanTile + threadIdx.x;
  int64_t v = (i < n) ? in[i] : 0;
  int64_t inc = block_incl_scan(v, sh);
  if (i < n) out[i] = sums[blockIdx.x] + inc - v;
  if (i == 0) out[n] = sums[tiles];
}

// Small inputs in one launch: thread t scans its run of ceil(n / 1024)
// consecutive counts, the block scans the run totals, then every run writes
// its offsets.
constexpr int64_t kScanOneBlock = 64 * 1024;
__global__ void scan_single_block(const int* __restrict__ in, int64_t n, int64_t* __restrict__ out) {
  __shared__ int64_t sh[32];
  const int64_t per = (n + kScanTile - 1) / kScanTile;
  const int64_t b = threadIdx.x * per, e = b + per < n ? b + per : n;
  int64_t tot = 0;
  for (int64_t i = b; i < e; ++i) tot += in[i];
  const int64_t inc = block_incl_scan(tot, sh);
  int64_t run = inc - tot;
  for (int64_t i = b; i < e; ++i) {
    out[i] = run;
    run += in[i];
  }
  if (threadIdx.x == kScanTile - 1) out[n] = inc;
}

size_t scan_tmp_elems(int64_t n) { return (size_t)((n + kScanTile - 1) / kScanTile + 1); }

int exclusive_scan_i32_to_i64(const int* in, int64_t* out, int64_t n, int64_t* tmp, cudaStream_t st) {
  if (n == 0) {
    cudaMemsetAsync(out, 0, sizeof(int64_t), st);
    return check_launch("scan(empty)", 0);
  }
  if (n <= kScanOneBlock) {
    scan_single_block<<<1, kScanTile, 0, st>>>(in, n, out);
    return check_launch("exclusive_scan");
  }
  int64_t tiles = (n + kScanTile - 1) / kScanTile;
  scan_tile_sums<<<(unsigned)tiles, kScanTile, 0, st>>>(in, n, tmp);
  scan_sums_serial<<<1, kScanTile, 0, st>>>(tmp, tiles);
  scan_apply<<<(unsigned)tiles, kScanTile, 0, st>>>(in, n, tmp, tiles, out);
  return check_launch("exclusive_scan", 3);
}

// ------------------------------------------------ device error flag / mode --
// Bounded device-side waits record a timeout here instead of hanging.
static __device__ int g_device_error;
static int* g_device_error_ptr[128] = {};
static void* g_device_error_ctx[128] = {};
static std::mutex g_flag_mu;
static std::atomic<int> g_mix_precision{0};

typedef int (*CtxGetCurrentFn)(void**);

void* current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(f);
  });
  void* ctx = nullptr;
  if (fn && fn(&ctx) != 0) ctx = nullptr;
  return ctx;
}

int* tc::error_flag() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return nullptr;
  void* ctx = current_context();
  std::lock_guard<std::mutex> lk(g_flag_mu);
  if (!g_device_error_ptr[dev] || g_device_error_ctx[dev] != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    g_device_error_ptr[dev] = static_cast<int*>(p);
    g_device_error_ctx[dev] = current_context();  // the lookup above made the context current
  }
  return g_device_error_ptr[dev];
}

int mix_precision() { return g_mix_precision.load(std::memory_order_relaxed); }

// ------------------------------------------------------- TMA descriptors --
// cuTensorMapEncodeTiled is a driver entry point; it is looked up once through
// the runtime so the library links against cudart only.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int tc::encode_tmap(CUtensorMap* map, const Operand& op, int box_inner, int box_outer, int swizzle) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  if (!fn) return set_error(BM_ERR_CUDA, "tc_gemm: cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(op.base) & 15) || (op.pitch & 15) || op.inner <= 0 || op.outer <= 0)
    return set_error(BM_ERR_INVALID_ARG, "tc_gemm: operand not 16-byte aligned (base %p, pitch %lld)", op.base,
                     (long long)op.pitch);
  const cuuint64_t dims[2] = {(cuuint64_t)op.inner, (cuuint64_t)op.outer};
  const cuuint64_t strides[1] = {(cuuint64_t)op.pitch};
  const cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(op.base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle == 2   ? CU_TENSOR_MAP_SWIZZLE_64B
                        : swizzle == 1 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                       : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(BM_ERR_CUDA, "tc_gemm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return BM_OK;
}

// --------------------------------------------------------- row sorting --
// One warp per row: every lane ranks its elements against the whole row
// (values in a row are distinct), then writes them to their rank.  Rows are
// staged through shared memory up to kSortStage entries; longer rows rank
// directly from global memory into a second half of the row buffer.
constexpr int kSortStage = 512;

__global__ void sort_rows_kernel(const int64_t* __restrict__ row_ptr, int64_t* __restrict__ vals,
                                 int64_t n_rows) {
  __shared__ int64_t stage[8][kSortStage];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t r = (int64_t)blockIdx.x * 8 + w;
  if (r >= n_rows) return;
  const int64_t b = row_ptr[r], d = row_ptr[r + 1] - b;
  if (d <= 1) return;
  int64_t* row = vals + b;
  if (d <= kSortStage) {
    for (int64_t k = lane; k < d; k += 32) stage[w][k] = row[k];
    __syncwarp();
    for (int64_t k = lane; k < d; k += 32) {
      const int64_t v = stage[w][k];
      int64_t rank = 0;
      for (int64_t q = 0; q < d; ++q) rank += (stage[w][q] < v);
      row[rank] = v;
    }
  } else {
    // Long row: odd-even transposition sort in place, warp-cooperative.
    for (int64_t phase = 0; phase < d; ++phase) {
      for (int64_t k = 2 * lane + (phase & 1); k + 1 < d; k += 64) {
        int64_t a = row[k], c = row[k + 1];
        if (a > c) { row[k] = c; row[k + 1] = a; }
      }
      __syncwarp();
    }
  }
}

int sort_rows_i64(const int64_t* row_ptr, int64_t* vals, int64_t n_rows, cudaStream_t st) {
  if (n_rows == 0) return BM_OK;
  sort_rows_kernel<<<grid_for(n_rows, 8), 256, 0, st>>>(row_ptr, vals, n_rows);
  return check_launch("sort_rows");
}

}  // namespace bm

extern "C" {

const char* bm_status_string(int s) {
  switch (s) {
    case BM_OK: return "ok";
    case BM_ERR_INVALID_ARG: return "invalid argument";
    case BM_ERR_CUDA: return "CUDA error";
    case BM_ERR_UNSUPPORTED: return "unsupported";
    case BM_ERR_CAPACITY: return "capacity exceeded";
    case BM_ERR_WORKSPACE: return "workspace too small";
    case BM_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

const char* bm_last_error(void) { return bm::g_last_error; }

int bm_version(void) { return 100; }

int64_t bm_launch_count(void) { return bm::g_launches.load(std::memory_order_relaxed); }

int bm_set_mix_precision(int mode) {
  BM_REQUIRE(mode == 0 || mode == 1, "bm_set_mix_precision: mode must be 0 (fp32) or 1 (tf32)");
  bm::g_mix_precision.store(mode);
  return BM_OK;
}

int bm_get_mix_precision(void) { return bm::mix_precision(); }

int bm_profile_start(void* stream) {
  std::lock_guard<std::mutex> lk(bm::g_prof_mu);
  for (auto& r : bm::g_prof_recs) bm::g_prof_pool.push_back(r.ev);
  bm::g_prof_recs.clear();
  bm::g_prof_totals.clear();
  bm::g_prof_stream = bm::as_stream(stream);
  bm::g_prof_on = true;
  bm::prof_record(nullptr);
  return BM_OK;
}

int bm_profile_mark(void) {
  std::lock_guard<std::mutex> lk(bm::g_prof_mu);
  if (bm::g_prof_on) bm::prof_record(nullptr);
  return BM_OK;
}

int bm_profile_stop(void) {
  std::lock_guard<std::mutex> lk(bm::g_prof_mu);
  if (!bm::g_prof_on) return BM_OK;
  bm::g_prof_on = false;
  cudaError_t e = cudaStreamSynchronize(bm::g_prof_stream);
  if (e != cudaSuccess) return bm::set_error(BM_ERR_CUDA, "bm_profile_stop: %s", cudaGetErrorString(e));
  for (size_t i = 1; i < bm::g_prof_recs.size(); ++i) {
    const auto& r = bm::g_prof_recs[i];
    if (!r.name) continue;
    float ms = 0.f;
    cudaEventElapsedTime(&ms, bm::g_prof_recs[i - 1].ev, r.ev);
    auto it = std::find_if(bm::g_prof_totals.begin(), bm::g_prof_totals.end(),
                           [&](const bm::ProfTotal& t) { return t.name == r.name; });
    if (it == bm::g_prof_totals.end()) bm::g_prof_totals.push_back({r.name, 1, ms});
    else { it->count += 1; it->ms += ms; }
  }
  return BM_OK;
}

int bm_profile_count(void) { return (int)bm::g_prof_totals.size(); }

int bm_profile_entry(int i, char* name, int name_len, int64_t* launches, double* total_ms) {
  BM_REQUIRE(i >= 0 && i < (int)bm::g_prof_totals.size() && name && name_len > 0, "bm_profile_entry: bad index");
  const auto& t = bm::g_prof_totals[i];
  snprintf(name, name_len, "%s", t.name.c_str());
  if (launches) *launches = t.count;
  if (total_ms) *total_ms = t.ms;
  return BM_OK;
}

int bm_device_error_check(void) {
  int* p = bm::tc::error_flag();
  if (!p) return bm::set_error(BM_ERR_CUDA, "bm_device_error_check: no device flag");
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && v != 0) {
    int z = 0;
    e = cudaMemcpy(p, &z, sizeof(int), cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) return bm::set_error(BM_ERR_CUDA, "bm_device_error_check: %s", cudaGetErrorString(e));
  // flag bits: 1 a bounded wait gave up, 2 an edge without its reverse in a
  // list taken as symmetric, 4 a neighbour-list fill given fewer edges than it found
  if (v & 1) return bm::set_error(BM_ERR_TIMEOUT, "a device-side wait timed out (pipelined kernel)");
  if (v & 4)
    return bm::set_error(BM_ERR_CAPACITY, "neighbor_list fill: the edge buffers hold fewer edges than the count "
                                          "found (positions changed since the count, or a short E); extra edges "
                                          "were dropped");
  if (v & 2) return bm::set_error(BM_ERR_INVALID_ARG, "csr_reverse: an edge has no reverse edge (list not symmetric)");
  return BM_OK;
}

int bm_tp_num_paths(void) { return bm::kNumPaths; }

int bm_tp_path_info(int32_t* out) {
  BM_REQUIRE(out != nullptr, "bm_tp_path_info: null output");
  for (int p = 0; p < bm::kNumPaths; ++p) {
    out[3 * p + 0] = bm::kPathL1[p];
    out[3 * p + 1] = bm::kPathL2[p];
    out[3 * p + 2] = bm::kPathLo[p];
  }
  return BM_OK;
}

}  // extern "C"

// ------------------------------------------------------------ fp32 probe --
// Peak fp32 FMA throughput of the device this process runs on, for the
// roofline of SIMT-bound kernels: every thread runs 8 independent FMA chains.
namespace bm {
__global__ void __launch_bounds__(256) fp32_probe_kernel(float* out, int iters, float a, float b) {
  float r[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) r[k] = threadIdx.x * 1e-3f + k;
  for (int i = 0; i < iters; ++i) {
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] = fmaf(r[k], a, b);
  }
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) s += r[k];
  if (s == 123.456f) out[0] = s;  // keeps the chains live
}
}  // namespace bm

extern "C" int bm_probe_fp32(float* scratch, int iters, int blocks, void* stream) {
  BM_REQUIRE(scratch && iters > 0 && blocks > 0, "bm_probe_fp32: bad arguments");
  bm::fp32_probe_kernel<<<blocks, 256, 0, bm::as_stream(stream)>>>(scratch, iters, 0.999f, 1e-4f);
  return bm::check_launch("bm_probe_fp32");
}

// -------------------------------------------------- tensor-core probe --
// Peak rate of the warp-level tf32 MMA (mma.sync m16n8k8, fp32 accumulate) on
// this device, the unit the edge-sum and target passes run on: every warp
// keeps 8 independent accumulators.
namespace bm {
__global__ void __launch_bounds__(256) mma_tf32_probe_kernel(float* out, int iters) {
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  const uint32_t l = threadIdx.x;
  const uint32_t a[4] = {__float_as_uint(1.0f + l), __float_as_uint(0.5f), __float_as_uint(0.25f), __float_as_uint(2.0f)};
  const uint32_t b0 = __float_as_uint(1e-3f), b1 = __float_as_uint(-1e-3f);
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) mma_tf32_16x8x8(acc[i], a, b0, b1);
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += acc[i][0] + acc[i][1] + acc[i][2] + acc[i][3];
  if (s == 123.456f) out[0] = s;  // keeps the chains live
}
}  // namespace bm

extern "C" int bm_probe_mma_tf32(float* scratch, int iters, int blocks, void* stream) {
  BM_REQUIRE(scratch && iters > 0 && blocks > 0, "bm_probe_mma_tf32: bad arguments");
  bm::mma_tf32_probe_kernel<<<blocks, 256, 0, bm::as_stream(stream)>>>(scratch, iters);
  return bm::check_launch("bm_probe_mma_tf32");
}

// ------------------------------------------------- bounded-wait self-test --
// One thread waits on a shared-memory mbarrier that nothing ever arrives on,
// through the same bounded wait every pipelined kernel of the library uses.
// The wait gives up after about a second, records the timeout in the device
// error flag and the kernel returns, so the context stays usable.
namespace bm {
__global__ void wait_timeout_selftest_kernel(int* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)tc::mbar_wait(&bar, 0, err);
  __syncthreads();
}
}  // namespace bm

extern "C" int bm_selftest_wait_timeout(void* stream) {
  int* err = bm::tc::error_flag();
  if (!err) return bm::set_error(BM_ERR_CUDA, "bm_selftest_wait_timeout: device error flag unavailable");
  cudaStream_t st = bm::as_stream(stream);
  bm::wait_timeout_selftest_kernel<<<1, 32, 0, st>>>(err);
  int rc = bm::check_launch("selftest(wait timeout)");
  if (rc) return rc;
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess)
    return bm::set_error(BM_ERR_CUDA, "bm_selftest_wait_timeout: %s", cudaGetErrorString(e));
  return bm_device_error_check();
}
