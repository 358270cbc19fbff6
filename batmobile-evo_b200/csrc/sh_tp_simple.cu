// Spherical harmonics forward/backward and the channel-free ("simple")
// tensor product.  All four are HBM-bound streaming kernels with one thread
// per edge/sample and every CG coefficient an immediate.  L = 3 (and the
// tensor products, which are L = 3 by construction) run as persistent
// TMA-staged kernels (namespace st below); other L_max, and SH calls whose
// inputs are not 16-byte aligned, use the one-block-per-256-edges kernels
// that stage their inputs through shared memory with 16-byte vector loads.
#include <mutex>

#include "bm_common.cuh"
#include "tc_gemm.cuh"

namespace bm {

constexpr int kBlk = 256;

// Stage `rows` x `w` floats of a dense row-major array into shared memory with
// float4 loads when the block's slice is 16-byte aligned (scalar otherwise).
__device__ __forceinline__ void stage_rows(const float* __restrict__ g, int64_t row0, int64_t nrows,
                                           int w, float* s) {
  const int64_t n = imin64(nrows - row0, kBlk) * w;
  const float* src = g + row0 * w;
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const int64_t n4 = n >> 2;
    for (int64_t k = threadIdx.x; k < n4; k += kBlk)
      reinterpret_cast<float4*>(s)[k] = __ldg(reinterpret_cast<const float4*>(src) + k);
    for (int64_t k = (n4 << 2) + threadIdx.x; k < n; k += kBlk) s[k] = __ldg(src + k);
  } else {
    for (int64_t k = threadIdx.x; k < n; k += kBlk) s[k] = __ldg(src + k);
  }
}

// [kBlk rows][16 floats] tile: float4 chunk c of row r at r * 4 + (c ^ ((r >> 1) & 3)),
// so both the one-row-per-thread writes (eight rows, eight distinct 16-byte
// banks) and the block-wide linear copy out (eight lanes = two whole rows per
// 128 bytes) are free of bank conflicts.
__device__ __forceinline__ int t16(int r, int c) { return r * 4 + (c ^ ((r >> 1) & 3)); }

__device__ __forceinline__ void tile_store16(float* __restrict__ g, int64_t row0, int rows, const float4* s) {
  float4* dst = reinterpret_cast<float4*>(g + row0 * 16);
  for (int k = threadIdx.x; k < rows * 4; k += kBlk) dst[k] = s[t16(k >> 2, k & 3)];
}
__device__ __forceinline__ void tile_put(float4* s, int r, const float* x) {
#pragma unroll
  for (int c = 0; c < 4; ++c) s[t16(r, c)] = make_float4(x[4 * c], x[4 * c + 1], x[4 * c + 2], x[4 * c + 3]);
}

template <int L>
__global__ void __launch_bounds__(kBlk) sh_fwd_kernel(const float* __restrict__ v, float* __restrict__ Y,
                                                      int64_t E) {
  constexpr int NC = (L + 1) * (L + 1);
  __shared__ __align__(16) float sv[kBlk * 3];
  const int64_t e0 = (int64_t)blockIdx.x * kBlk;
  stage_rows(v, e0, E, 3, sv);
  __syncthreads();
  const int64_t e = e0 + threadIdx.x;
  if constexpr (NC == 16) {  // L = 3: rows out through a tile
    __shared__ float4 so[kBlk * 4];
    const int rows = (int)imin64(E - e0, kBlk);
    if (e < E) {
      float o[16];
      sh_eval<L>(sv[3 * threadIdx.x], sv[3 * threadIdx.x + 1], sv[3 * threadIdx.x + 2], o);
      tile_put(so, threadIdx.x, o);
    }
    __syncthreads();
    tile_store16(Y, e0, rows, so);
    return;
  }
  if (e >= E) return;
  float o[NC];
  sh_eval<L>(sv[3 * threadIdx.x], sv[3 * threadIdx.x + 1], sv[3 * threadIdx.x + 2], o);
  float* dst = Y + e * NC;
  if (NC % 4 == 0) {
#pragma unroll
    for (int k = 0; k < NC / 4; ++k)
      reinterpret_cast<float4*>(dst)[k] = make_float4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
  } else {
#pragma unroll
    for (int k = 0; k < NC; ++k) dst[k] = o[k];
  }
}

template <int L>
__global__ void __launch_bounds__(kBlk) sh_bwd_kernel(const float* __restrict__ v, const float* __restrict__ gY,
                                                      float* __restrict__ gv, int64_t E) {
  constexpr int NC = (L + 1) * (L + 1);
  __shared__ __align__(16) float sv[kBlk * 3];
  __shared__ __align__(16) float so[kBlk * 3];
  const int64_t e0 = (int64_t)blockIdx.x * kBlk;
  stage_rows(v, e0, E, 3, sv);
  __syncthreads();
  const int64_t e = e0 + threadIdx.x;
  if (e < E) {
    float g[NC];
    const float* src = gY + e * NC;
    if (NC % 4 == 0 && (reinterpret_cast<uintptr_t>(gY) & 15) == 0) {
#pragma unroll
      for (int k = 0; k < NC / 4; ++k) {
        float4 q = __ldg(reinterpret_cast<const float4*>(src) + k);
        g[4 * k] = q.x; g[4 * k + 1] = q.y; g[4 * k + 2] = q.z; g[4 * k + 3] = q.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < NC; ++k) g[k] = __ldg(src + k);
    }
    float gx, gy, gz;
    const float x = sv[3 * threadIdx.x], y = sv[3 * threadIdx.x + 1], z = sv[3 * threadIdx.x + 2];
    if constexpr (L <= 3) {
      sh_grad<L>(x, y, z, g, gx, gy, gz);
    } else {
      // l = 4..6: the recurrence evaluated on dual numbers (exact Jacobian)
      D3 o[NC];
      sh_eval<L, D3>(D3(x, 1.0f, 0.0f, 0.0f), D3(y, 0.0f, 1.0f, 0.0f), D3(z, 0.0f, 0.0f, 1.0f), o);
      gx = gy = gz = 0.0f;
#pragma unroll
      for (int k = 1; k < NC; ++k) {
        gx = fmaf(g[k], o[k].dx, gx);
        gy = fmaf(g[k], o[k].dy, gy);
        gz = fmaf(g[k], o[k].dz, gz);
      }
    }
    so[3 * threadIdx.x] = gx; so[3 * threadIdx.x + 1] = gy; so[3 * threadIdx.x + 2] = gz;
  }
  __syncthreads();
  const int64_t n = imin64(E - e0, kBlk) * 3;
  for (int64_t k = threadIdx.x; k < n; k += kBlk) gv[e0 * 3 + k] = so[k];
}

__device__ __forceinline__ void store16(float* p, const float* r) {
#pragma unroll
  for (int k = 0; k < 4; ++k)
    reinterpret_cast<float4*>(p)[k] = make_float4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]);
}

// ---------------------------------------------------------------------------
// Persistent TMA-staged versions of the L = 3 streaming ops (the case every
// caller of the irreps layout uses).  Each CTA of kST threads walks tiles of
// kST edges; per tile the [E, 16] operands arrive as one 2D TMA box each
// (SWIZZLE_64B: 16-byte chunk c of row r at chunk c ^ ((r >> 1) & 3), so one
// thread per row reads its 64 bytes without bank conflicts) and [E, 3] edge
// vectors as one 1D bulk copy, into a ring of kSS stages completing on
// mbarriers; the next tiles' copies are in flight while a tile is computed.
// The SH forward writes its rows into a swizzled tile stored by TMA; the
// other outputs go straight from registers.  Arithmetic is the same code, in
// the same order, as the one-thread-per-edge kernels above, so the results
// are identical bit for bit.
namespace st {

constexpr int kST = 128;                      // edges per tile = consumer threads per CTA
constexpr int kCW = kST / 32;                 // consumer warps
constexpr int kThreads = kST + 32;            // + one producer warp
constexpr uint32_t kTile16 = kST * 16 * 4;    // one [kST, 16] fp32 box (8 KB)
constexpr uint32_t kTileV = kST * 3 * 4;      // one [kST, 3] fp32 slice (1536 B)
// Input stages, chosen by measurement on the B200 at 1M edges (64- and
// 256-row tiles, and other depths, measured slower).
constexpr int kSSsh = 3;                      // SH forward and backward
constexpr int kSSfw = 2;                      // tensor product forward (6 CTAs per SM)
constexpr int kSSbw = 3;                      // tensor product backward (3 CTAs per SM)

__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void tma_store_nocommit(const CUtensorMap* map, int x, int y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}

// Row r of a swizzled [kST, 16] tile into registers.
__device__ __forceinline__ void ld_row16(const float* tile, int r, float* o) {
  const float4* t = reinterpret_cast<const float4*>(tile) + r * 4;
  const int sw = (r >> 1) & 3;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 q = t[c ^ sw];
    o[4 * c] = q.x; o[4 * c + 1] = q.y; o[4 * c + 2] = q.z; o[4 * c + 3] = q.w;
  }
}
__device__ __forceinline__ void st_row16(float* tile, int r, const float* o) {
  float4* t = reinterpret_cast<float4*>(tile) + r * 4;
  const int sw = (r >> 1) & 3;
#pragma unroll
  for (int c = 0; c < 4; ++c) t[c ^ sw] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
}

struct Maps {
  CUtensorMap in[3];   // [E, 16] inputs (SWIZZLE_64B boxes of kST rows)
  CUtensorMap out;     // SH forward output
};

// Shared-memory plan: kSS input stages of (NI x 8 KB boxes, then the edge-vector
// slice when HV), then (SH forward) two output tiles, then the mbarriers.
template <int NI, bool HV, bool TOUT, int kSS>
struct Plan {
  static constexpr uint32_t kStage = NI * kTile16 + (HV ? kTileV : 0);
  static constexpr uint32_t kStageP = (kStage + 1023) & ~1023u;
  static constexpr uint32_t kOut = kSS * kStageP;
  static constexpr uint32_t kBar = kOut + (TOUT ? 2 * kTile16 : 0);
  static constexpr uint32_t kBytes = kBar + 2 * 8 * kSS + 1024;   // + alignment slack
};

// Issues the copies of tile `t` into stage `s` (one thread).
template <int NI, bool HV, bool TOUT, int kSS>
__device__ __forceinline__ void issue(uint8_t* sm, int s, int64_t t, const Maps& M, const float* v, int64_t E,
                                      uint64_t* bar) {
  using P = Plan<NI, HV, TOUT, kSS>;
  uint8_t* st = sm + s * P::kStageP;
  const int64_t e0 = t * kST;
  uint32_t vbytes = 0;
  if (HV) vbytes = (uint32_t)((imin64(E - e0, kST) * 12) & ~int64_t(15));   // whole 16-byte units
  tc::mbar_expect_tx(bar, NI * kTile16 + vbytes);
#pragma unroll
  for (int i = 0; i < NI; ++i) tc::tma_load_2d(tc::smem_u32(st + i * kTile16), &M.in[i], 0, (int)e0, bar);
  if (HV && vbytes) tc::bulk_g2s(st + NI * kTile16, v + e0 * 3, vbytes, bar);
}

// The persistent tile loop, warp-specialised: warp kCW (the last) is the
// producer, which refills a stage as soon as the kCW consumer warps have
// released it; each consumer thread owns one row of every tile.
// body(e, r, valid, in_tiles, vx, vy, vz, out_tile) runs once per consumer
// thread per tile (r = row in the tile, e = global edge, valid = e < E).
// The SH forward's output rows go out per warp: each consumer warp stores its
// 32 rows of the (double-buffered) output tile with its own TMA store.
template <int NI, bool HV, bool TOUT, int kSS, class Body>
__device__ __forceinline__ void tile_loop(const Maps& M, const float* __restrict__ v, int64_t E, int* err, Body body) {
  using P = Plan<NI, HV, TOUT, kSS>;
  extern __shared__ uint8_t st_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(st_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + P::kBar);
  uint64_t* empty = full + kSS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t ntiles = (E + kST - 1) / kST;
  if (tid == 0) {
    for (int s = 0; s < kSS; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], kCW);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == kCW) {   // producer
    if (lane == 0) {
      int it = 0;
      for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int s = it % kSS;
        if (it >= kSS && !tc::mbar_wait(&empty[s], (uint32_t)((it / kSS - 1) & 1), err)) break;
        issue<NI, HV, TOUT, kSS>(sm, s, t, M, v, E, &full[s]);
      }
    }
    return;
  }
  int it = 0;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
    const int s = it % kSS;
    if (TOUT && lane == 0) bulk_wait_read1();   // this warp's store of two tiles ago has read its rows
    const bool ok = tc::mbar_wait(&full[s], (uint32_t)((it / kSS) & 1), err);
    if (!__all_sync(0xffffffffu, ok)) break;   // the whole warp leaves together on a timeout
    uint8_t* stg = sm + s * P::kStageP;
    const int64_t e0 = t * kST;
    const int64_t e = e0 + tid;
    const bool valid = e < E;
    float vx = 0.0f, vy = 0.0f, vz = 0.0f;
    if (HV && valid) {
      const float* vs = reinterpret_cast<const float*>(stg + NI * kTile16);
      const uint32_t have = (uint32_t)((imin64(E - e0, kST) * 12) & ~int64_t(15)) / 4;   // floats copied
      if ((uint32_t)(3 * tid + 2) < have) {
        vx = vs[3 * tid]; vy = vs[3 * tid + 1]; vz = vs[3 * tid + 2];
      } else {   // the ragged end of the last tile
        vx = __ldg(v + 3 * e); vy = __ldg(v + 3 * e + 1); vz = __ldg(v + 3 * e + 2);
      }
    }
    float* otile = TOUT ? reinterpret_cast<float*>(sm + P::kOut + (it & 1) * kTile16) : nullptr;
    body(e, tid, valid, reinterpret_cast<const float*>(stg), vx, vy, vz, otile);
    if (TOUT) tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tc::mbar_arrive(&empty[s]);   // this warp is done with stage s
      if (TOUT && e0 + warp * 32 < E) {
        tma_store_nocommit(&M.out, 0, (int)(e0 + warp * 32), tc::smem_u32(otile + warp * 32 * 16));
        bulk_commit();
      }
    }
  }
  if (TOUT && lane == 0) tc::bulk_wait0();
}

__global__ void __launch_bounds__(kThreads) sh3_fwd_kernel(const __grid_constant__ Maps M, const float* __restrict__ v,
                                                    int64_t E, int* err) {
  tile_loop<0, true, true, kSSsh>(M, v, E, err,
                           [&](int64_t, int r, bool valid, const float*, float x, float y, float z, float* ot) {
                             float o[16];
                             sh_eval<3>(x, y, z, o);
                             if (!valid) {
#pragma unroll
                               for (int k = 0; k < 16; ++k) o[k] = 0.0f;
                             }
                             st_row16(ot, r, o);
                           });
}

__global__ void __launch_bounds__(kThreads) sh3_bwd_kernel(const __grid_constant__ Maps M, const float* __restrict__ v,
                                                    float* __restrict__ gv, int64_t E, int* err) {
  tile_loop<1, true, false, kSSsh>(M, v, E, err,
                            [&](int64_t e, int r, bool valid, const float* in, float x, float y, float z, float*) {
                              if (!valid) return;
                              float g[16];
                              ld_row16(in, r, g);
                              float gx, gy, gz;
                              sh_grad<3>(x, y, z, g, gx, gy, gz);
                              gv[3 * e] = gx; gv[3 * e + 1] = gy; gv[3 * e + 2] = gz;
                            });
}

__global__ void __launch_bounds__(kThreads) tp_fwd_kernel(const __grid_constant__ Maps M, float* __restrict__ out,
                                                   int64_t N, int* err) {
  tile_loop<2, false, false, kSSfw>(M, nullptr, N, err,
                             [&](int64_t n, int r, bool valid, const float* in, float, float, float, float*) {
                               if (!valid) return;
                               float x[16], y[16], o[16];
                               ld_row16(in, r, x);
                               ld_row16(in + kST * 16, r, y);
#pragma unroll
                               for (int k = 0; k < 16; ++k) o[k] = 0.0f;
#define BM_X(p, m1, m2, mo, c) o[mo] = fmaf(c, x[m1] * y[m2], o[mo]);
                               BM_CG_ALL(BM_X)
#undef BM_X
                               store16(out + n * 16, o);
                             });
}

__global__ void __launch_bounds__(kThreads, 3) tp_bwd_kernel(const __grid_constant__ Maps M, float* __restrict__ ga,
                                                   float* __restrict__ gb, int64_t N, int* err) {
  tile_loop<3, false, false, kSSbw>(M, nullptr, N, err,
                             [&](int64_t n, int r, bool valid, const float* in, float, float, float, float*) {
                               if (!valid) return;
                               float x[16], y[16], go[16], dx[16], dy[16];
                               ld_row16(in, r, x);
                               ld_row16(in + kST * 16, r, y);
                               ld_row16(in + 2 * kST * 16, r, go);
#pragma unroll
                               for (int k = 0; k < 16; ++k) { dx[k] = 0.0f; dy[k] = 0.0f; }
#define BM_X(p, m1, m2, mo, c)                  \
  dx[m1] = fmaf(c, go[mo] * y[m2], dx[m1]);     \
  dy[m2] = fmaf(c, go[mo] * x[m1], dy[m2]);
                               BM_CG_ALL(BM_X)
#undef BM_X
                               if (ga) store16(ga + n * 16, dx);
                               if (gb) store16(gb + n * 16, dy);
                             });
}

// [rows, 16] fp32 map with kST-row SWIZZLE_64B boxes.
static int map16(CUtensorMap* m, const float* p, int64_t rows, int box_rows = kST) {
  tc::Operand op{p, 16, rows, 64};
  return tc::encode_tmap(m, op, 16, box_rows, 2);
}

// Persistent grid of a kernel at `smem` dynamic bytes: resident CTAs per SM
// times the SM count (cached per kernel `id` and device), at most `ntiles`.
template <class K>
static int grid_of(int id, K kernel, uint32_t smem, int64_t ntiles, int* rc) {
  static std::mutex mu;
  static int cache[4][128] = {};
  int* cached = cache[id];
  int dev = 0;
  *rc = BM_OK;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) dev = 0;
  int per_sm;
  {
    std::lock_guard<std::mutex> lk(mu);
    per_sm = cached[dev];
  }
  if (per_sm == 0) {
    cudaError_t e = cudaFuncSetAttribute((const void*)kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int sms = kNumSMs, occ = 0;
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kThreads, smem);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess || occ <= 0) {
      *rc = set_error(BM_ERR_CUDA, "streaming kernel set-up: %s", cudaGetErrorString(e));
      return 0;
    }
    per_sm = occ * sms;
    std::lock_guard<std::mutex> lk(mu);
    cached[dev] = per_sm;
  }
  return (int)imin64(ntiles, per_sm);
}

static int launch_sh3_fwd(const float* v, float* Y, int64_t E, cudaStream_t stream) {
  using P = Plan<0, true, true, kSSsh>;
  Maps M;
  int rc = map16(&M.out, Y, E, 32);
  if (rc) return rc;
  const int g = grid_of(0, sh3_fwd_kernel, P::kBytes, (E + kST - 1) / kST, &rc);
  if (rc) return rc;
  sh3_fwd_kernel<<<g, kThreads, P::kBytes, stream>>>(M, v, E, tc::error_flag());
  return check_launch("spherical_harmonics");
}

static int launch_sh3_bwd(const float* v, const float* gY, float* gv, int64_t E, cudaStream_t stream) {
  using P = Plan<1, true, false, kSSsh>;
  Maps M;
  int rc = map16(&M.in[0], gY, E);
  if (rc) return rc;
  const int g = grid_of(1, sh3_bwd_kernel, P::kBytes, (E + kST - 1) / kST, &rc);
  if (rc) return rc;
  sh3_bwd_kernel<<<g, kThreads, P::kBytes, stream>>>(M, v, gv, E, tc::error_flag());
  return check_launch("spherical_harmonics_backward");
}

static int launch_tp_fwd(const float* a, const float* b, float* out, int64_t N, cudaStream_t stream) {
  using P = Plan<2, false, false, kSSfw>;
  Maps M;
  int rc = map16(&M.in[0], a, N);
  if (!rc) rc = map16(&M.in[1], b, N);
  if (rc) return rc;
  const int g = grid_of(2, tp_fwd_kernel, P::kBytes, (N + kST - 1) / kST, &rc);
  if (rc) return rc;
  tp_fwd_kernel<<<g, kThreads, P::kBytes, stream>>>(M, out, N, tc::error_flag());
  return check_launch("tensor_product_simple");
}

static int launch_tp_bwd(const float* a, const float* b, const float* go, float* ga, float* gb, int64_t N,
                         cudaStream_t stream) {
  using P = Plan<3, false, false, kSSbw>;
  Maps M;
  int rc = map16(&M.in[0], a, N);
  if (!rc) rc = map16(&M.in[1], b, N);
  if (!rc) rc = map16(&M.in[2], go, N);
  if (rc) return rc;
  const int g = grid_of(3, tp_bwd_kernel, P::kBytes, (N + kST - 1) / kST, &rc);
  if (rc) return rc;
  tp_bwd_kernel<<<g, kThreads, P::kBytes, stream>>>(M, ga, gb, N, tc::error_flag());
  return check_launch("tensor_product_simple_backward");
}

}  // namespace st

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace bm

using namespace bm;

extern "C" {

int bm_sh_fwd(const float* v, float* Y, int64_t E, int L, void* stream) {
  BM_REQUIRE(L >= 0 && L <= 6, "spherical_harmonics: L_max must be in [0, 6], got %d", L);
  BM_REQUIRE(E >= 0, "spherical_harmonics: negative edge count");
  if (E == 0) return BM_OK;
  BM_REQUIRE(v && Y, "spherical_harmonics: null pointer");
  const int NC = (L + 1) * (L + 1);
  BM_REQUIRE(NC % 4 != 0 || aligned16(Y), "spherical_harmonics: output must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  if (L == 3 && aligned16(v)) return st::launch_sh3_fwd(v, Y, E, st);
  unsigned g = grid_for(E, kBlk);
  switch (L) {
    case 0: sh_fwd_kernel<0><<<g, kBlk, 0, st>>>(v, Y, E); break;
    case 1: sh_fwd_kernel<1><<<g, kBlk, 0, st>>>(v, Y, E); break;
    case 2: sh_fwd_kernel<2><<<g, kBlk, 0, st>>>(v, Y, E); break;
    case 3: sh_fwd_kernel<3><<<g, kBlk, 0, st>>>(v, Y, E); break;
    case 4: sh_fwd_kernel<4><<<g, kBlk, 0, st>>>(v, Y, E); break;
    case 5: sh_fwd_kernel<5><<<g, kBlk, 0, st>>>(v, Y, E); break;
    case 6: sh_fwd_kernel<6><<<g, kBlk, 0, st>>>(v, Y, E); break;
  }
  return check_launch("spherical_harmonics");
}

int bm_sh_bwd(const float* v, const float* gY, float* gv, int64_t E, int L, void* stream) {
  BM_REQUIRE(L >= 0 && L <= 6, "spherical_harmonics_backward: invalid L_max %d", L);
  if (E == 0) return BM_OK;
  BM_REQUIRE(v && gY && gv, "spherical_harmonics_backward: null pointer");
  cudaStream_t st = as_stream(stream);
  if (L == 3 && aligned16(v) && aligned16(gY)) return st::launch_sh3_bwd(v, gY, gv, E, st);
  unsigned g = grid_for(E, kBlk);
  switch (L) {
    case 0: sh_bwd_kernel<0><<<g, kBlk, 0, st>>>(v, gY, gv, E); break;
    case 1: sh_bwd_kernel<1><<<g, kBlk, 0, st>>>(v, gY, gv, E); break;
    case 2: sh_bwd_kernel<2><<<g, kBlk, 0, st>>>(v, gY, gv, E); break;
    case 3: sh_bwd_kernel<3><<<g, kBlk, 0, st>>>(v, gY, gv, E); break;
    case 4: sh_bwd_kernel<4><<<g, kBlk, 0, st>>>(v, gY, gv, E); break;
    case 5: sh_bwd_kernel<5><<<g, kBlk, 0, st>>>(v, gY, gv, E); break;
    case 6: sh_bwd_kernel<6><<<g, kBlk, 0, st>>>(v, gY, gv, E); break;
  }
  return check_launch("spherical_harmonics_backward");
}

int bm_tp_simple_fwd(const float* a, const float* b, float* out, int64_t N, void* stream) {
  BM_REQUIRE(N >= 0, "tensor_product_simple: negative N");
  if (N == 0) return BM_OK;
  BM_REQUIRE(a && b && out, "tensor_product_simple: null pointer");
  BM_REQUIRE(aligned16(a) && aligned16(b) && aligned16(out),
             "tensor_product_simple: tensors must be 16-byte aligned");
  return st::launch_tp_fwd(a, b, out, N, as_stream(stream));
}

int bm_tp_simple_bwd(const float* a, const float* b, const float* g, float* ga, float* gb, int64_t N,
                     void* stream) {
  BM_REQUIRE(N >= 0, "tensor_product_simple_backward: negative N");
  if (N == 0) return BM_OK;
  BM_REQUIRE(a && b && g, "tensor_product_simple_backward: null pointer");
  BM_REQUIRE(aligned16(a) && aligned16(b) && aligned16(g) && (!ga || aligned16(ga)) && (!gb || aligned16(gb)),
             "tensor_product_simple_backward: tensors must be 16-byte aligned");
  if (!ga && !gb) return BM_OK;
  return st::launch_tp_bwd(a, b, g, ga, gb, N, as_stream(stream));
}

}  // extern "C"
