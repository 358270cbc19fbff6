// Graph-side kernels: COO -> CSR by target (deterministic), the reference's
// unweighted fused SH+TP message kernel, segmented (atomics-free) message
// passing, and the reduction of per-edge vector gradients onto atoms.
#include "mix_gemm.cuh"

namespace bm {

// ------------------------------------------------------------------- CSR --
__global__ void csr_count_kernel(const int64_t* __restrict__ dst, int64_t E, int64_t N, int* __restrict__ cnt) {
  int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  int64_t d = dst[e];
  if (d >= 0 && d < N) atomicAdd(cnt + d, 1);
}

__global__ void csr_fill_kernel(const int64_t* __restrict__ dst, int64_t E, int64_t N,
                                const int64_t* __restrict__ row_ptr, int* __restrict__ cursor,
                                int64_t* __restrict__ col_idx) {
  int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= E) return;
  int64_t d = dst[e];
  if (d < 0 || d >= N) return;
  int slot = atomicAdd(cursor + d, 1);
  col_idx[row_ptr[d] + slot] = e;  // order fixed afterwards by sort_rows
}

// -------------------------------------------- unweighted fused SH + TP --
__device__ __forceinline__ void tp16_acc(const float* x, const float* y, float* o) {
#define BM_X(p, m1, m2, mo, c) o[mo] = fmaf(c, x[m1] * y[m2], o[mo]);
  BM_CG_ALL(BM_X)
#undef BM_X
}

__device__ __forceinline__ void ld16(const float* __restrict__ p, float* r) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float4 q = __ldg(reinterpret_cast<const float4*>(p) + k);
    r[4 * k] = q.x; r[4 * k + 1] = q.y; r[4 * k + 2] = q.z; r[4 * k + 3] = q.w;
  }
}
__device__ __forceinline__ void st16(float* p, const float* r) {
#pragma unroll
  for (int k = 0; k < 4; ++k)
    reinterpret_cast<float4*>(p)[k] = make_float4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]);
}

__global__ void __launch_bounds__(256) fused_sh_tp_simple_kernel(const float* __restrict__ v, const float* __restrict__ x,
                                                                 const int64_t* __restrict__ src, float* __restrict__ msg,
                                                                 int64_t E, int64_t N, int C) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= E * C) return;
  const int64_t e = t / C;
  const int c = (int)(t - e * C);
  float y[16], xv[16], o[16];
  sh_eval<3>(__ldg(v + 3 * e), __ldg(v + 3 * e + 1), __ldg(v + 3 * e + 2), y);
  const int64_t s = src[e];
  if (s < 0 || s >= N) {
#pragma unroll
    for (int k = 0; k < 16; ++k) o[k] = 0.0f;
  } else {
    ld16(x + (s * C + c) * 16, xv);
#pragma unroll
    for (int k = 0; k < 16; ++k) o[k] = 0.0f;
    tp16_acc(xv, y, o);
  }
  st16(msg + t * 16, o);
}

// out[n, c] = sum over CSR row n of TP_simple(x[source, c], Y(v[edge])) in row
// order.  kSrcFromCol: col_idx holds the source atom and v is in CSR order
// (weighted-binding contract); otherwise col_idx holds edge ids and the source
// is edge_index[0][e].
template <bool kSrcFromCol>
__global__ void __launch_bounds__(128) mp_simple_kernel(const float* __restrict__ x, const float* __restrict__ v,
                                                        const int64_t* __restrict__ edge_src,
                                                        const int64_t* __restrict__ row_ptr,
                                                        const int64_t* __restrict__ col_idx, float* __restrict__ out,
                                                        int64_t N, int C) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= N * C) return;
  const int64_t n = t / C;
  const int c = (int)(t - n * C);
  float o[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) o[k] = 0.0f;
  const int64_t b = row_ptr[n], e_end = row_ptr[n + 1];
  for (int64_t k = b; k < e_end; ++k) {
    const int64_t ci = col_idx[k];
    const int64_t e = kSrcFromCol ? k : ci;
    const int64_t s = kSrcFromCol ? ci : edge_src[ci];
    if (s < 0 || s >= N) continue;
    float y[16], xv[16];
    sh_eval<3>(__ldg(v + 3 * e), __ldg(v + 3 * e + 1), __ldg(v + 3 * e + 2), y);
    ld16(x + (s * C + c) * 16, xv);
    tp16_acc(xv, y, o);
  }
  st16(out + t * 16, o);
}

// W2p[co][ci] = W2[ci][co] with the ci pitch padded to a multiple of 4 (zeros).
__global__ void pack_w2_kernel(const float* __restrict__ W2, int Ci, int Co, int CPi, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)Co * CPi) return;
  const int co = (int)(i / CPi), ci = (int)(i - (int64_t)co * CPi);
  out[i] = ci < Ci ? W2[(int64_t)ci * Co + co] : 0.0f;
}

// grad_pos[n] = sum_{e: dst=n} gv[e] - sum_{e: src=n} gv[e].  One warp per atom:
// lane l sums the row entries l, l + 32, ... of both rows, then a fixed shuffle
// tree adds the lanes (deterministic order).
__global__ void edge_grad_to_pos_kernel(const float* __restrict__ gv, const int64_t* __restrict__ rpd,
                                        const int64_t* __restrict__ pd, const int64_t* __restrict__ rps,
                                        const int64_t* __restrict__ ps, float* __restrict__ gp, int64_t N) {
  const int64_t n = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  float ax = 0.f, ay = 0.f, az = 0.f;
  for (int64_t k = rpd[n] + lane; k < rpd[n + 1]; k += 32) {
    const int64_t e = pd[k];
    ax += gv[3 * e]; ay += gv[3 * e + 1]; az += gv[3 * e + 2];
  }
  for (int64_t k = rps[n] + lane; k < rps[n + 1]; k += 32) {
    const int64_t e = ps[k];
    ax -= gv[3 * e]; ay -= gv[3 * e + 1]; az -= gv[3 * e + 2];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ax += __shfl_xor_sync(0xffffffffu, ax, o);
    ay += __shfl_xor_sync(0xffffffffu, ay, o);
    az += __shfl_xor_sync(0xffffffffu, az, o);
  }
  if (lane == 0) { gp[3 * n] = ax; gp[3 * n + 1] = ay; gp[3 * n + 2] = az; }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Reverse-edge index of a symmetric CSR whose rows are sorted: for the entry k
// of row i holding column j, rev[k] = position of i inside row j (binary
// search).  rev is then the target-grouped permutation of the edge list
// (row_ptr serves both orders), and rev[rev[k]] == k.  One warp per row, so
// the row of an entry is known without a search; a missing reverse edge
// writes -1 and raises the device error flag.
__global__ void csr_reverse_kernel(const int64_t* __restrict__ row_ptr, const int64_t* __restrict__ col, int64_t N,
                                   int64_t* __restrict__ rev, int* err) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= N) return;
  const int64_t kb = row_ptr[i], ke = row_ptr[i + 1];
  for (int64_t k = kb + lane; k < ke; k += 32) {
    const int64_t j = col[k];
    int64_t r = -1;
    if (j >= 0 && j < N) {
      int64_t a = row_ptr[j], b = row_ptr[j + 1];
      const int64_t end = b;
      while (a < b) {
        const int64_t mid = (a + b) >> 1;
        if (col[mid] < i) a = mid + 1; else b = mid;
      }
      if (a < end && col[a] == i) r = a;
    }
    rev[k] = r;
    if (r < 0) atomicOr(err, 2);
  }
}

}  // namespace bm

using namespace bm;

extern "C" {

size_t bm_csr_workspace_bytes(int64_t N, int64_t) {
  return sizeof(int) * 2 * (size_t)(N + 4) + sizeof(int64_t) * scan_tmp_elems(N + 1) + 256;
}

int bm_edge_index_to_csr(const int64_t* ei, int64_t* row_ptr, int64_t* col_idx, int64_t N, int64_t E, void* ws,
                         size_t ws_bytes, void* stream) {
  BM_REQUIRE(N >= 0 && E >= 0, "edge_index_to_csr: negative size");
  BM_REQUIRE(E < (int64_t(1) << 31), "edge_index_to_csr: more than 2^31 edges");
  BM_REQUIRE(row_ptr != nullptr, "edge_index_to_csr: null row_ptr");
  cudaStream_t st = as_stream(stream);
  if (E == 0) {
    cudaMemsetAsync(row_ptr, 0, sizeof(int64_t) * (N + 1), st);
    return check_launch("edge_index_to_csr(empty)", 0);
  }
  BM_REQUIRE(ei && col_idx, "edge_index_to_csr: null pointer");
  if (!ws || ws_bytes < bm_csr_workspace_bytes(N, E))
    return set_error(BM_ERR_WORKSPACE, "edge_index_to_csr: workspace too small");
  int* cnt = static_cast<int*>(ws);
  int* cursor = cnt + (N + 4);
  int64_t* tmp = reinterpret_cast<int64_t*>(
      (reinterpret_cast<uintptr_t>(cursor + (N + 4)) + 15) & ~uintptr_t(15));
  cudaMemsetAsync(cnt, 0, sizeof(int) * 2 * (size_t)(N + 4), st);
  const int64_t* dst = ei + E;
  csr_count_kernel<<<grid_for(E, 256), 256, 0, st>>>(dst, E, N, cnt);
  int rc = check_launch("edge_index_to_csr(count)");
  if (rc) return rc;
  if ((rc = exclusive_scan_i32_to_i64(cnt, row_ptr, N, tmp, st))) return rc;
  csr_fill_kernel<<<grid_for(E, 256), 256, 0, st>>>(dst, E, N, row_ptr, cursor, col_idx);
  if ((rc = check_launch("edge_index_to_csr(fill)"))) return rc;
  return sort_rows_i64(row_ptr, col_idx, N, st);
}

int bm_csr_reverse(const int64_t* row_ptr, const int64_t* col, int64_t N, int64_t E, int64_t* rev, void* stream) {
  BM_REQUIRE(N >= 0 && E >= 0, "csr_reverse: negative size");
  if (E == 0) return BM_OK;
  BM_REQUIRE(row_ptr && col && rev, "csr_reverse: null pointer");
  int* err = tc::error_flag();
  if (!err) return set_error(BM_ERR_CUDA, "csr_reverse: device error flag unavailable");
  csr_reverse_kernel<<<grid_for(N * 32, 256), 256, 0, as_stream(stream)>>>(row_ptr, col, N, rev, err);
  return check_launch("csr_reverse");
}

int bm_fused_sh_tp_simple(const float* v, const float* x, const int64_t* src, float* msg, int64_t E, int64_t N,
                          int C, void* stream) {
  BM_REQUIRE(E >= 0 && N >= 0 && C > 0, "fused_sh_tp_simple: bad sizes");
  if (E == 0) return BM_OK;
  BM_REQUIRE(v && x && src && msg, "fused_sh_tp_simple: null pointer");
  BM_REQUIRE(al16(x) && al16(msg), "fused_sh_tp_simple: tensors must be 16-byte aligned");
  fused_sh_tp_simple_kernel<<<grid_for(E * C, 256), 256, 0, as_stream(stream)>>>(v, x, src, msg, E, N, C);
  return check_launch("fused_sh_tp_simple");
}

int bm_fused_mp_simple(const float* x, const float* v, const int64_t* ei, const int64_t* row_ptr,
                       const int64_t* col_idx, float* out, int64_t N, int64_t E, int C, void* stream) {
  BM_REQUIRE(N >= 0 && E >= 0 && C > 0, "fused_message_passing_simple: bad sizes");
  if (N == 0) return BM_OK;
  BM_REQUIRE(x && out && row_ptr && (E == 0 || (v && ei && col_idx)), "fused_message_passing_simple: null pointer");
  BM_REQUIRE(al16(x) && al16(out), "fused_message_passing_simple: tensors must be 16-byte aligned");
  mp_simple_kernel<false><<<grid_for(N * C, 128), 128, 0, as_stream(stream)>>>(x, v, ei, row_ptr, col_idx, out, N, C);
  return check_launch("fused_message_passing_simple");
}

size_t bm_fused_mp_weighted_workspace_bytes(int64_t N, int Ci, int Co) {
  return sizeof(float) * ((size_t)N * Ci * 16 + (size_t)N * 16 * pitch4(Ci) + (size_t)Co * pitch4(Ci));
}

int bm_fused_mp_weighted(const float* x, const float* v, const float* W2, const int64_t* row_ptr,
                         const int64_t* col_idx, float* out, int64_t N, int64_t E, int Ci, int Co, void* ws,
                         size_t ws_bytes, void* stream) {
  BM_REQUIRE(N >= 0 && E >= 0 && Ci > 0 && Co > 0, "fused_message_passing: bad sizes");
  if (N == 0) return BM_OK;
  BM_REQUIRE(x && W2 && out && row_ptr && (E == 0 || (v && col_idx)), "fused_message_passing: null pointer");
  BM_REQUIRE(al16(x) && al16(out), "fused_message_passing: tensors must be 16-byte aligned");
  if (!ws || ws_bytes < bm_fused_mp_weighted_workspace_bytes(N, Ci, Co))
    return set_error(BM_ERR_WORKSPACE, "fused_message_passing: workspace too small");
  cudaStream_t st = as_stream(stream);
  float* T = static_cast<float*>(ws);
  mp_simple_kernel<true><<<grid_for(N * Ci, 128), 128, 0, st>>>(x, v, nullptr, row_ptr, col_idx, T, N, Ci);
  int rc = check_launch("fused_message_passing(aggregate)");
  if (rc) return rc;
  // out[n, co, m] = sum_ci T[n, ci, m] W2[ci, co] as a tensor-core GEMM over rows (n, m)
  const int CPi = pitch4(Ci);
  float* Tt = T + (size_t)N * Ci * 16;
  float* W2p = Tt + (size_t)N * 16 * CPi;
  if ((rc = pack_irreps(T, N, Ci, 0, 16, Tt, st))) return rc;
  pack_w2_kernel<<<grid_for((int64_t)Co * CPi, 256), 256, 0, st>>>(W2, Ci, Co, CPi, W2p);
  if ((rc = check_launch("fused_message_passing(pack)"))) return rc;
  MixOut p{Tt, N * 16, CPi, W2p, Co, out, 16, 0};
  return run_mix(p, st);
}

int bm_edge_grad_to_pos(const float* gv, const int64_t* rpd, const int64_t* pd, const int64_t* rps,
                        const int64_t* ps, float* gp, int64_t N, void* stream) {
  BM_REQUIRE(N >= 0, "edge_grad_to_pos: bad size");
  if (N == 0) return BM_OK;
  BM_REQUIRE(gv && rpd && pd && rps && ps && gp, "edge_grad_to_pos: null pointer");
  edge_grad_to_pos_kernel<<<grid_for(N * 32, 256), 256, 0, as_stream(stream)>>>(gv, rpd, pd, rps, ps, gp, N);
  return check_launch("edge_grad_to_pos");
}

}  // extern "C"
