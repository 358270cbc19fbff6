// Weighted 34-path tensor product (reference: src/tensor_product/tensor_product.cu:133-201,
// tensor_product_backward.cu:948-1005):
//
//   out[n, co, mo] = sum_p sum_ci W[p, ci, co] sum_{(m1,m2,mo) in p} c x[n, ci, m1] Y[n, m2]
//
// Split into a per-(sample, channel) CG stage that writes the slot array
// S[g][(n, m)][(pos, ci)] (156 values per channel, grouped by l_out) and one
// grouped mixing GEMM per l_out -- instead of redoing the 611-term CG for every
// output channel as the reference does.
#include "mix_gemm.cuh"

namespace bm {

__global__ void sum_splits_kernel(const float* __restrict__ part, int64_t stride, int splits,
                                  float* __restrict__ out, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.0f;
  for (int k = 0; k < splits; ++k) s += part[k * stride + i];
  out[i] = s;
}

int sum_splits(const float* part, int64_t stride, int splits, float* out, int64_t n, cudaStream_t st) {
  if (n == 0) return BM_OK;
  sum_splits_kernel<<<grid_for(n, 256), 256, 0, st>>>(part, stride, splits, out, n);
  return check_launch("sum_splits");
}

// Store the CG contraction of one channel into its l_out-grouped slots.
// S layout per group g: [(n*(2g+1) + m) * P_g + pos] * CP + c  (CP = channel pitch).
#define BM_SLOT_LO(p, m1, m2, mo, c)                                                   \
  if constexpr (kPathLo[p] == G) {                                                    \
    constexpr int I_ = ((mo) - G * G) * kGroupPaths[G] + kPathPosLo[p];               \
    acc[I_] = fmaf((c), x[m1] * y[m2], acc[I_]);                                      \
  }

template <int G>
__device__ __forceinline__ void cg_slots_group(const float* x, const float* y, float* S, int64_t N,
                                               int64_t n, int CP, int c) {
  constexpr int P = kGroupPaths[G];
  constexpr int R = (2 * G + 1) * P;
  float acc[R];
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = 0.0f;
  BM_CG_ALL(BM_SLOT_LO)
  float* base = S + N * CP * (int64_t)kGroupSlotOff[G] + n * (int64_t)R * CP + c;
#pragma unroll
  for (int i = 0; i < R; ++i) base[(int64_t)i * CP] = acc[i];
}

// One thread per (sample, padded channel); padding channels write zeros.
__global__ void __launch_bounds__(128) tp_slots_kernel(const float* __restrict__ x, const float* __restrict__ Y,
                                                       float* __restrict__ S, int64_t N, int C, int CP) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= N * CP) return;
  const int64_t n = t / CP;
  const int c = (int)(t - n * CP);
  float xv[16], yv[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    xv[k] = c < C ? __ldg(x + (n * C + c) * 16 + k) : 0.0f;
    yv[k] = __ldg(Y + n * 16 + k);
  }
  cg_slots_group<0>(xv, yv, S, N, n, CP, c);
  cg_slots_group<1>(xv, yv, S, N, n, CP, c);
  cg_slots_group<2>(xv, yv, S, N, n, CP, c);
  cg_slots_group<3>(xv, yv, S, N, n, CP, c);
}

// Backward CG stage: from dS (l_out-grouped slots, pitch CP), per (sample, ci):
//   gx[n, ci, m1] = sum c dS[p, mo] Y[m2],   gYpart[n, ci, m2] = sum c dS[p, mo] x[m1]
__global__ void __launch_bounds__(128) tp_bwd_cg_kernel(const float* __restrict__ x, const float* __restrict__ Y,
                                                        const float* __restrict__ dS, float* __restrict__ gx,
                                                        float* __restrict__ gy_part, int64_t N, int C, int CP) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= N * C) return;
  const int64_t n = t / C;
  const int c = (int)(t - n * C);
  float xv[16], yv[16], dx[16], dy[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    xv[k] = __ldg(x + t * 16 + k); yv[k] = __ldg(Y + n * 16 + k); dx[k] = 0.0f; dy[k] = 0.0f;
  }
#define BM_BWD(p, m1, m2, mo, cf)                                                                   \
  { constexpr int G_ = kPathLo[p];                                                                 \
    constexpr int OFF_ = kGroupSlotOff[G_], P_ = kGroupPaths[G_], POS_ = kPathPosLo[p];              \
    const float s_ = __ldg(dS + N * CP * (int64_t)OFF_ +                                             \
                           ((n * (2 * G_ + 1) + ((mo) - G_ * G_)) * P_ + POS_) * CP + c);             \
    dx[m1] = fmaf((cf) * s_, yv[m2], dx[m1]);                                                      \
    dy[m2] = fmaf((cf) * s_, xv[m1], dy[m2]); }
  BM_CG_ALL(BM_BWD)
#undef BM_BWD
  if (gx) {
#pragma unroll
    for (int k = 0; k < 16; ++k) gx[t * 16 + k] = dx[k];
  }
  if (gy_part) {
#pragma unroll
    for (int k = 0; k < 16; ++k) gy_part[t * 16 + k] = dy[k];
  }
}

// gY[n, m] = sum_ci gy_part[n, ci, m]  (fixed order: deterministic)
__global__ void reduce_channels_kernel(const float* __restrict__ part, float* __restrict__ out, int64_t N, int C) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= N * 16) return;
  const int64_t n = t >> 4;
  const int m = (int)(t & 15);
  float s = 0.0f;
  for (int c = 0; c < C; ++c) s += part[(n * C + c) * 16 + m];
  out[t] = s;
}

// ------------------------------------------------------------- packing --
struct PackArgs {
  int path[4][11];
  int64_t off[5];
  int P[4];
};

__global__ void pack_weights_kernel(const float* __restrict__ W, int Ci, int Co, int mode, PackArgs a,
                                    float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.off[4]) return;
  int g = 0;
  while (g < 3 && i >= a.off[g + 1]) ++g;
  // every packed group holds fewer than 2^32 entries (checked by pack_weights),
  // so the index arithmetic below runs in 32 bits
  const unsigned j = (unsigned)(i - a.off[g]);
  const unsigned CPi = (Ci + 3) & ~3, CPo = (Co + 3) & ~3, P = a.P[g];
  int pos, ci, co;
  if (mode == kPackFwd) {          // [co][pos*CPi + ci]
    const unsigned row = j / (P * CPi), col = j - row * (P * CPi);
    co = (int)row; pos = (int)(col / CPi); ci = (int)(col - pos * CPi);
  } else if (mode == kPackDx) {    // [ci][pos*CPo + co]
    const unsigned row = j / (P * CPo), col = j - row * (P * CPo);
    ci = (int)row; pos = (int)(col / CPo); co = (int)(col - pos * CPo);
  } else {                         // [pos*CPi + ci][co]
    const unsigned row = j / CPo;
    co = (int)(j - row * CPo); pos = (int)(row / CPi); ci = (int)(row - pos * CPi);
  }
  out[i] = (ci < Ci && co < Co) ? W[((int64_t)a.path[g][pos] * Ci + ci) * Co + co] : 0.0f;
}

int pack_weights(const float* W, int Ci, int Co, int mode, float* out, cudaStream_t st) {
  PackArgs a{};
  for (int g = 0; g < 4; ++g) {
    a.P[g] = kGroupPaths[g];
    for (int i = 0; i < 11; ++i) a.path[g][i] = mode == kPackDx ? kL1Group[g][i] : kLoGroup[g][i];
  }
  for (int g = 0; g <= 4; ++g) a.off[g] = pack_group_offset(mode, g, Ci, Co);
  for (int g = 0; g < 4; ++g)
    BM_REQUIRE(a.off[g + 1] - a.off[g] < (int64_t(1) << 32), "pack_weights: C_in = %d, C_out = %d too large", Ci, Co);
  pack_weights_kernel<<<grid_for(a.off[4], 256), 256, 0, st>>>(W, Ci, Co, mode, a, out);
  return check_launch("pack_weights");
}

__global__ void pack_irreps_kernel(const float* __restrict__ G, int64_t N, int C, int CP, int comp0, int cnt,
                                   float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N * cnt * CP) return;
  const int64_t row = i / CP;
  const int c = (int)(i - row * CP);
  const int64_t n = row / cnt;
  const int m = (int)(row - n * cnt);
  out[i] = c < C ? __ldg(G + (n * C + c) * 16 + comp0 + m) : 0.0f;
}

int pack_irreps(const float* G, int64_t N, int C, int comp0, int cnt, float* out, cudaStream_t st) {
  const int CP = pitch4(C);
  if (N == 0) return BM_OK;
  pack_irreps_kernel<<<grid_for(N * cnt * CP, 256), 256, 0, st>>>(G, N, C, CP, comp0, cnt, out);
  return check_launch("pack_irreps");
}

// All four l-groups in one pass: thread (n, c) reads G[n, c, 0:16] (one
// contiguous 64-byte row) and writes component m of group g to
// out[N g^2 CP + (n (2g+1) + m - g^2) CP + c]; consecutive threads are
// consecutive channels, so both sides are coalesced.
__global__ void pack_irreps_groups_kernel(const float* __restrict__ G, int64_t N, int C, int CP,
                                          float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N * CP) return;
  const int64_t n = i / CP;
  const int c = (int)(i - n * CP);
  float v[16];
  if (c < C) {
    const float4* src = reinterpret_cast<const float4*>(G + (n * C + c) * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 a = __ldg(src + q);
      v[4 * q] = a.x; v[4 * q + 1] = a.y; v[4 * q + 2] = a.z; v[4 * q + 3] = a.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = 0.0f;
  }
#pragma unroll
  for (int g = 0; g < 4; ++g)
#pragma unroll
    for (int m = 0; m < 2 * g + 1; ++m)
      out[N * (int64_t)(g * g) * CP + (n * (2 * g + 1) + m) * CP + c] = v[g * g + m];
}

int pack_irreps_groups(const float* G, int64_t N, int C, float* out, cudaStream_t st) {
  if (N == 0) return BM_OK;
  const int CP = pitch4(C);
  if ((reinterpret_cast<uintptr_t>(G) & 15) != 0) {  // unaligned input: per-group gathers
    for (int g = 0; g < 4; ++g) {
      const int rc = pack_irreps(G, N, C, g * g, 2 * g + 1, out + (size_t)N * g * g * CP, st);
      if (rc) return rc;
    }
    return BM_OK;
  }
  pack_irreps_groups_kernel<<<grid_for(N * CP, 256), 256, 0, st>>>(G, N, C, CP, out);
  return check_launch("pack_irreps");
}

static size_t slots_floats(int64_t N, int C) { return (size_t)N * pitch4(C) * kSlots; }

// Forward: CG slots, then one tensor-core mix per l_out group.  S holds
// slots_floats(N, Ci); Wf holds pack_floats(kPackFwd, Ci, Co).
static int tp_forward(const float* x, const float* Y, const float* W, float* out, int64_t N, int Ci, int Co,
                      float* S, float* Wf, cudaStream_t st) {
  const int CPi = pitch4(Ci);
  int rc = pack_weights(W, Ci, Co, kPackFwd, Wf, st);
  if (rc) return rc;
  tp_slots_kernel<<<grid_for(N * CPi, 128), 128, 0, st>>>(x, Y, S, N, Ci, CPi);
  if ((rc = check_launch("tensor_product(cg)"))) return rc;
  MixOut ps[4];
  for (int g = 0; g < 4; ++g)
    ps[g] = MixOut{S + slot_group_offset(g, N, CPi), N * (2 * g + 1), (int64_t)kGroupPaths[g] * CPi,
                   Wf + pack_group_offset(kPackFwd, g, Ci, Co), Co, out, 2 * g + 1, g * g};
  return run_mix4(ps, st);
}

}  // namespace bm

using namespace bm;

extern "C" {

size_t bm_tp_fwd_workspace_bytes(int64_t N, int Ci, int Co) {
  return (slots_floats(N, Ci) + (size_t)pack_floats(kPackFwd, Ci, Co)) * sizeof(float);
}

int bm_tp_fwd(const float* x, const float* Y, const float* W, float* out, int64_t N, int Ci, int Co,
              void* ws, size_t ws_bytes, void* stream) {
  BM_REQUIRE(N >= 0 && Ci > 0 && Co > 0, "tensor_product: bad sizes N=%lld C_in=%d C_out=%d", (long long)N, Ci, Co);
  if (N == 0) return BM_OK;
  BM_REQUIRE(x && Y && W && out, "tensor_product: null pointer");
  if (ws_bytes < bm_tp_fwd_workspace_bytes(N, Ci, Co) || !ws)
    return set_error(BM_ERR_WORKSPACE, "tensor_product: workspace too small");
  float* S = static_cast<float*>(ws);
  return tp_forward(x, Y, W, out, N, Ci, Co, S, S + slots_floats(N, Ci), as_stream(stream));
}

size_t bm_tp_bwd_workspace_bytes(int64_t N, int Ci, int Co) {
  size_t f = 2 * slots_floats(N, Ci) + (size_t)N * Ci * 16 + (size_t)N * 16 * pitch4(Co) +
             (size_t)pack_floats(kPackDs, Ci, Co) + (size_t)kMaxSplits * kNumPaths * Ci * Co;
  return f * sizeof(float);
}

int bm_tp_bwd(const float* x, const float* Y, const float* W, const float* G, float* gx, float* gY, float* gW,
              int64_t N, int Ci, int Co, void* ws, size_t ws_bytes, void* stream) {
  BM_REQUIRE(N >= 0 && Ci > 0 && Co > 0, "tensor_product_backward: bad sizes");
  cudaStream_t st = as_stream(stream);
  if (N == 0) {
    if (gW) cudaMemsetAsync(gW, 0, sizeof(float) * kNumPaths * Ci * Co, st);
    return check_launch("tensor_product_backward(empty)", 0);
  }
  BM_REQUIRE(x && Y && W && G, "tensor_product_backward: null pointer");
  if (ws_bytes < bm_tp_bwd_workspace_bytes(N, Ci, Co) || !ws)
    return set_error(BM_ERR_WORKSPACE, "tensor_product_backward: workspace too small");
  const int CPi = pitch4(Ci), CPo = pitch4(Co);
  float* S = static_cast<float*>(ws);
  float* dS = S + slots_floats(N, Ci);
  float* gyp = dS + slots_floats(N, Ci);
  float* Gt = gyp + (size_t)N * Ci * 16;            // [g blocks of N(2g+1) rows][CPo]
  float* Ws = Gt + (size_t)N * 16 * CPo;
  float* part = Ws + pack_floats(kPackDs, Ci, Co);
  int rc;
  if ((rc = pack_irreps_groups(G, N, Co, Gt, st))) return rc;
  if (gW) {
    tp_slots_kernel<<<grid_for(N * CPi, 128), 128, 0, st>>>(x, Y, S, N, Ci, CPi);
    if ((rc = check_launch("tensor_product_backward(cg)"))) return rc;
    const int64_t stride = (int64_t)kNumPaths * Ci * Co;
    const int splits = dw_splits_all(N, Ci, Co);
    MixWeights ps[4];
    for (int g = 0; g < 4; ++g)
      ps[g] = MixWeights{S + slot_group_offset(g, N, CPi), kGroupPaths[g] * CPi, N * (2 * g + 1),
                   Gt + (size_t)N * g * g * CPo, CPo, Co, lo_group(g), Ci, CPi, part, stride};
    if ((rc = run_mix4(ps, st, splits))) return rc;
    if ((rc = sum_splits(part, stride, splits, gW, stride, st))) return rc;
  }
  if (gx || gY) {
    if ((rc = pack_weights(W, Ci, Co, kPackDs, Ws, st))) return rc;
    MixSlots ps[4];
    for (int g = 0; g < 4; ++g)
      ps[g] = MixSlots{Gt + (size_t)N * g * g * CPo, N * (2 * g + 1), CPo, Ws + pack_group_offset(kPackDs, g, Ci, Co),
                 kGroupPaths[g] * CPi, dS + slot_group_offset(g, N, CPi)};
    if ((rc = run_mix4(ps, st))) return rc;
    tp_bwd_cg_kernel<<<grid_for(N * Ci, 128), 128, 0, st>>>(x, Y, dS, gx, gY ? gyp : nullptr, N, Ci, CPi);
    if ((rc = check_launch("tensor_product_backward(cg^T)"))) return rc;
    if (gY) {
      reduce_channels_kernel<<<grid_for(N * 16, 256), 256, 0, st>>>(gyp, gY, N, Ci);
      if ((rc = check_launch("tensor_product_backward(reduce)"))) return rc;
    }
  }
  return BM_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// bm_tp_fwd_noalloc: the weighted tensor product without caller workspace.
//
// Some callers cannot hand this library device scratch: a host program that
// binds the plain C ABI through a foreign-function layer with no device
// allocator of its own, or a simulation loop that reserves all device memory
// up front and must not call cudaMalloc mid-step (it can synchronise the device
// and break the step's time budget).  For them this entry point keeps its
// scratch -- the per-sample CG slot array (N * 156 floats per input channel,
// channels padded to a multiple of 4) and a repacked copy of the weights -- in a
// fixed-size array in the library's own device memory, so a call allocates
// nothing.  The array costs kNoAllocScratchFloats * 4 bytes on every GPU that
// loads the library, for the life of the process.
//
// Sharing: every call uses the same array.  Each call overwrites all slots it
// reads before reading them (nothing needs to start at zero), but two calls
// that overlap on the GPU (different streams, or different host threads
// without ordering) race on the array and produce wrong results.
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress while that device is current; make that first call
// before any stream capture.  The address is cached per device together with
// the CUDA context it belongs to, and looked up again when the context changes
// (after cudaDeviceReset, for instance).
// ---------------------------------------------------------------------------
#include <mutex>

namespace bm {

constexpr size_t kNoAllocScratchFloats = size_t(6) << 20;  // 24 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[128] = {};
static void* g_noalloc_ctx[128] = {};

static int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(BM_ERR_CUDA, "tensor_product_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 128) return set_error(BM_ERR_UNSUPPORTED, "tensor_product_noalloc: device %d", dev);
  void* ctx = current_context();
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev] || g_noalloc_ctx[dev] != ctx) {  // first call, or a new context after a reset
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(BM_ERR_CUDA, "tensor_product_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<float*>(p);
    g_noalloc_ctx[dev] = current_context();
  }
  *out = g_noalloc_ptr[dev];
  return BM_OK;
}

}  // namespace bm

extern "C" {

size_t bm_tp_fwd_noalloc_max_floats(void) { return bm::kNoAllocScratchFloats; }

int bm_tp_fwd_noalloc(const float* x, const float* Y, const float* W, float* out, int64_t N, int Ci, int Co,
                      void* stream) {
  BM_REQUIRE(N >= 0 && Ci > 0 && Co > 0, "tensor_product_noalloc: bad sizes N=%lld C_in=%d C_out=%d",
             (long long)N, Ci, Co);
  if (N == 0) return BM_OK;
  BM_REQUIRE(x && Y && W && out, "tensor_product_noalloc: null pointer");
  const size_t need = bm_tp_fwd_workspace_bytes(N, Ci, Co) / sizeof(float);
  if (need > kNoAllocScratchFloats)
    return set_error(BM_ERR_CAPACITY,
                     "tensor_product_noalloc: needs %zu scratch floats (N * 156 per padded input channel plus "
                     "the packed weights), which exceeds the fixed scratch of %zu floats (24 MiB); use bm_tp_fwd "
                     "with a caller workspace", need, kNoAllocScratchFloats);
  float* S = nullptr;
  int rc = noalloc_scratch(&S);
  if (rc) return rc;
  return tp_forward(x, Y, W, out, N, Ci, Co, S, S + slots_floats(N, Ci), as_stream(stream));
}

}  // extern "C"
