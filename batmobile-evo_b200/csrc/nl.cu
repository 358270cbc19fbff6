// Periodic cell-list neighbour list with a bit-exact, deterministic,
// lexicographically sorted edge set; orthorhombic boxes and general
// (triclinic) cells.
//
// Predicate (per ordered pair i != j), evaluated in fp32 with every operation
// rounded on its own (no FMA contraction), identical to the reference's
// brute-force check benchmarks/benchmark_neighbor_list_standalone.py:110-125:
//   d = p_i - p_j;  d -= rint(d / L) * L  (per axis, true division);
//   s = (dx*dx + dy*dy) + dz*dz;  keep if s <= float(cutoff^2).
// Cells: nb = floor(L / (cutoff * (1 + 1e-4))) per axis (at least 3), so every
// cell is wider than the cutoff with a margin larger than fp32 rounding and the
// 27 surrounding cells hold every candidate (with nb = 3 they are the whole box).
//
// Triclinic cells (rows of H = lattice vectors a, b, c; positions p = s H):
// the same predicate with the minimum image taken in fractional coordinates,
//   s = d Hinv;  s -= rint(s);  d = s H   (row-vector products, each sum
//   left to right, every operation rounded on its own),
// Hinv = inverse(H) in float64 rounded to fp32.  Atoms are binned by their
// wrapped fractional coordinates; the bins per lattice direction are
// floor(h / (cutoff * (1 + 1e-4))) (at least 3) with h the cell's
// perpendicular height along that direction, so a pair within the cutoff
// differs by at most one bin per direction.  A cell whose off-diagonal
// entries are all zero takes the orthorhombic path above, bit for bit.
//
// Passes: bin (atomic slot per cell) -> scan -> scatter atoms into cell order
// -> count per atom -> scan = row_ptr -> write unsorted targets -> per-row rank
// sort, i written, vectors p_j - p_i min-imaged.  Nothing reads the atomic
// order, so the output is deterministic.
#include <cmath>
#include <cstring>

#include "bm_common.cuh"

namespace bm {
namespace tc {
int* error_flag();  // device error flag of the current device (api.cu)
}
}  // namespace bm

namespace bm {

struct NLGeom {
  float L[3];
  int nb[3];
  int ncell;
  float rc2;
  int64_t n_rows;  // only atoms i < n_rows get rows (all atoms are candidates)
  int tri;         // 1: general cell H (row-major, rows = lattice vectors), Hi = inverse
  float H[9], Hi[9];
};

static int nl_geom(const float* box, double cutoff, NLGeom& g) {
  g.tri = 0;
  if (!box) return set_error(BM_ERR_INVALID_ARG, "neighbor_list: null box");
  if (!(cutoff > 0.0)) return set_error(BM_ERR_INVALID_ARG, "neighbor_list: cutoff must be > 0");
  int64_t total = 1;
  for (int a = 0; a < 3; ++a) {
    if (!(box[a] > 0.0f) || !std::isfinite(box[a]))
      return set_error(BM_ERR_INVALID_ARG, "neighbor_list: box lengths must be positive and finite");
    g.L[a] = box[a];
    double n = std::floor((double)box[a] / (cutoff * (1.0 + 1e-4)));
    if (n < 3) n = 3;
    if (n > 1024) n = 1024;
    g.nb[a] = (int)n;
    total *= g.nb[a];
  }
  if (total > (int64_t(1) << 28)) return set_error(BM_ERR_CAPACITY, "neighbor_list: too many cells");
  g.ncell = (int)total;
  g.rc2 = (float)(cutoff * cutoff);
  g.n_rows = INT64_MAX;
  return BM_OK;
}

// Geometry from a host float[9] cell (row-major, rows = lattice vectors).
static int nl_geom_cell(const float* cell, double cutoff, NLGeom& g) {
  if (!cell) return set_error(BM_ERR_INVALID_ARG, "neighbor_list: null cell");
  for (int k = 0; k < 9; ++k)
    if (!std::isfinite(cell[k])) return set_error(BM_ERR_INVALID_ARG, "neighbor_list: cell entries must be finite");
  if (cell[1] == 0.0f && cell[2] == 0.0f && cell[3] == 0.0f && cell[5] == 0.0f && cell[6] == 0.0f && cell[7] == 0.0f) {
    const float box[3] = {cell[0], cell[4], cell[8]};
    return nl_geom(box, cutoff, g);
  }
  if (!(cutoff > 0.0)) return set_error(BM_ERR_INVALID_ARG, "neighbor_list: cutoff must be > 0");
  double h[9];
  for (int k = 0; k < 9; ++k) h[k] = cell[k];
  // cofactors: row k of the inverse's transpose is (row a x row b) / det
  double cr[3][3];
  for (int k = 0; k < 3; ++k) {
    const double* a = h + 3 * ((k + 1) % 3);
    const double* b = h + 3 * ((k + 2) % 3);
    cr[k][0] = a[1] * b[2] - a[2] * b[1];
    cr[k][1] = a[2] * b[0] - a[0] * b[2];
    cr[k][2] = a[0] * b[1] - a[1] * b[0];
  }
  const double det = h[0] * cr[0][0] + h[1] * cr[0][1] + h[2] * cr[0][2];
  const double norm = std::sqrt(h[0] * h[0] + h[1] * h[1] + h[2] * h[2]) *
                      std::sqrt(h[3] * h[3] + h[4] * h[4] + h[5] * h[5]) *
                      std::sqrt(h[6] * h[6] + h[7] * h[7] + h[8] * h[8]);
  if (!(std::fabs(det) > 1e-6 * norm))
    return set_error(BM_ERR_INVALID_ARG, "neighbor_list: cell vectors are (nearly) linearly dependent");
  int64_t total = 1;
  for (int k = 0; k < 3; ++k) {
    const double area = std::sqrt(cr[k][0] * cr[k][0] + cr[k][1] * cr[k][1] + cr[k][2] * cr[k][2]);
    const double height = std::fabs(det) / area;  // distance between the lattice planes of direction k
    double n = std::floor(height / (cutoff * (1.0 + 1e-4)));
    if (n < 3) n = 3;
    if (n > 1024) n = 1024;
    g.nb[k] = (int)n;
    total *= g.nb[k];
    g.L[k] = (float)height;
  }
  if (total > (int64_t(1) << 28)) return set_error(BM_ERR_CAPACITY, "neighbor_list: too many cells");
  // Hinv[m][k] = cr[k][m] / det  (row-vector convention s = p Hinv)
  for (int m = 0; m < 3; ++m)
    for (int k = 0; k < 3; ++k) g.Hi[3 * m + k] = (float)(cr[k][m] / det);
  for (int k = 0; k < 9; ++k) g.H[k] = cell[k];
  g.tri = 1;
  g.ncell = (int)total;
  g.rc2 = (float)(cutoff * cutoff);
  g.n_rows = INT64_MAX;
  return BM_OK;
}

// Component k of the row-vector product (x, y, z) M for a row-major 3x3 M.
__device__ __forceinline__ float rowvec3(float x, float y, float z, const float* M, int k) {
  return __fadd_rn(__fadd_rn(__fmul_rn(x, M[k]), __fmul_rn(y, M[3 + k])), __fmul_rn(z, M[6 + k]));
}

// Fractional-coordinate minimum image of a Cartesian difference (triclinic cells).
__device__ __forceinline__ void min_image_tri(float& dx, float& dy, float& dz, const NLGeom& g) {
  float s0 = rowvec3(dx, dy, dz, g.Hi, 0), s1 = rowvec3(dx, dy, dz, g.Hi, 1), s2 = rowvec3(dx, dy, dz, g.Hi, 2);
  s0 = __fsub_rn(s0, rintf(s0));
  s1 = __fsub_rn(s1, rintf(s1));
  s2 = __fsub_rn(s2, rintf(s2));
  dx = rowvec3(s0, s1, s2, g.H, 0);
  dy = rowvec3(s0, s1, s2, g.H, 1);
  dz = rowvec3(s0, s1, s2, g.H, 2);
}

// Bin of a fractional coordinate along one lattice direction.
__device__ __forceinline__ int frac_bin(float s, int nb) {
  const float w = __fsub_rn(s, floorf(s));
  const int c = (int)floorf(__fmul_rn(w, (float)nb));
  return min(max(c, 0), nb - 1);
}

__device__ __forceinline__ int cell_coord(float p, float L, int nb) {
  float w = __fsub_rn(p, __fmul_rn(floorf(__fdiv_rn(p, L)), L));
  int c = (int)floorf(__fdiv_rn(__fmul_rn(w, (float)nb), L));
  return min(max(c, 0), nb - 1);
}

__device__ __forceinline__ float min_image(float d, float L) {
  return __fsub_rn(d, __fmul_rn(rintf(__fdiv_rn(d, L)), L));
}

__device__ __forceinline__ bool pair_within(float4 pi, float4 pj, const NLGeom& g) {
  float dx, dy, dz;
  if (g.tri) {
    dx = __fsub_rn(pi.x, pj.x);
    dy = __fsub_rn(pi.y, pj.y);
    dz = __fsub_rn(pi.z, pj.z);
    min_image_tri(dx, dy, dz, g);
  } else {
    dx = min_image(__fsub_rn(pi.x, pj.x), g.L[0]);
    dy = min_image(__fsub_rn(pi.y, pj.y), g.L[1]);
    dz = min_image(__fsub_rn(pi.z, pj.z), g.L[2]);
  }
  float s = __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
  return s <= g.rc2;
}

__global__ void nl_bin_kernel(const float* __restrict__ pos, int64_t N, NLGeom g, int* __restrict__ cell_of,
                              int* __restrict__ slot_of, int* __restrict__ cell_cnt) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  const float px = pos[3 * i], py = pos[3 * i + 1], pz = pos[3 * i + 2];
  int cx, cy, cz;
  if (g.tri) {
    cx = frac_bin(rowvec3(px, py, pz, g.Hi, 0), g.nb[0]);
    cy = frac_bin(rowvec3(px, py, pz, g.Hi, 1), g.nb[1]);
    cz = frac_bin(rowvec3(px, py, pz, g.Hi, 2), g.nb[2]);
  } else {
    cx = cell_coord(px, g.L[0], g.nb[0]);
    cy = cell_coord(py, g.L[1], g.nb[1]);
    cz = cell_coord(pz, g.L[2], g.nb[2]);
  }
  int c = (cz * g.nb[1] + cy) * g.nb[0] + cx;
  cell_of[i] = c;
  slot_of[i] = atomicAdd(cell_cnt + c, 1);
}

__global__ void nl_scatter_kernel(const float* __restrict__ pos, int64_t N, const int* __restrict__ cell_of,
                                  const int* __restrict__ slot_of, const int64_t* __restrict__ cell_start,
                                  int* __restrict__ sorted_idx, float4* __restrict__ sorted_pos) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= N) return;
  int64_t k = cell_start[cell_of[i]] + slot_of[i];
  sorted_idx[k] = (int)i;
  sorted_pos[k] = make_float4(pos[3 * i], pos[3 * i + 1], pos[3 * i + 2], 0.0f);
}

// Candidate ranges of the 27 cells around cell c in the cell-sorted atom order:
// the three cells x-1, x, x+1 of each of the 9 (y, z) rows are adjacent in that
// order, so a row is one contiguous range, or two where it wraps around the
// periodic x boundary (x = 0 or x = nb-1).  Lane r < 18 gets part r & 1 of
// row r >> 1 as [b, e) (empty where the row needs one range only, and for
// lanes 18..31).
__device__ __forceinline__ void lane_range(int c, const NLGeom& g, const int64_t* __restrict__ cell_start, int lane,
                                           int64_t& b, int64_t& e) {
  b = e = 0;
  if (lane >= 18) return;
  const int nx = g.nb[0];
  const int cx = c % nx;
  const int cy = (c / nx) % g.nb[1];
  const int cz = c / (nx * g.nb[1]);
  const int rw = lane >> 1, part = lane & 1;
  int z = cz + rw / 3 - 1; z += (z < 0) ? g.nb[2] : 0; z -= (z >= g.nb[2]) ? g.nb[2] : 0;
  int y = cy + rw % 3 - 1; y += (y < 0) ? g.nb[1] : 0; y -= (y >= g.nb[1]) ? g.nb[1] : 0;
  const int row = (z * g.nb[1] + y) * nx;
  int c0, c1;   // cells [c0, c1) of this part
  if (cx == 0) {                 // cells nx-1 | 0, 1
    c0 = part ? row + nx - 1 : row;
    c1 = part ? row + nx : row + 2;
  } else if (cx == nx - 1) {     // cells nx-2, nx-1 | 0
    c0 = part ? row : row + nx - 2;
    c1 = part ? row + 1 : row + nx;
  } else {
    if (part) return;
    c0 = row + cx - 1;
    c1 = row + cx + 2;
  }
  b = cell_start[c0];
  e = cell_start[c1];
}

// One warp per atom (atoms in cell order for locality).  The candidates of
// the up to 18 ranges are numbered 0..T-1 in range order; pass p hands
// candidate 32p + lane to each lane (range found by a binary search over the
// lanes' running totals), and the next pass's loads are issued before this
// pass's distance checks, so a row costs about one memory latency per pass
// rather than two per range.  Matches are counted with ballots and, in the
// write pass, compacted to ballot-prefix positions (the row is sorted
// afterwards, so the order here is irrelevant).
template <bool kWrite, class IdxT>
__global__ void __launch_bounds__(128) nl_pairs_kernel(int64_t N, NLGeom g, bool self_loops,
                                                       const int* __restrict__ cell_of,
                                                       const int64_t* __restrict__ cell_start,
                                                       const int* __restrict__ sorted_idx,
                                                       const float4* __restrict__ sorted_pos,
                                                       int* __restrict__ cnt, const int64_t* __restrict__ row_ptr,
                                                       IdxT* __restrict__ tmp_j, int64_t E, int* __restrict__ err) {
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int64_t k = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (k >= N) return;
  const int i = sorted_idx[k];
  if (i >= g.n_rows) {
    if (!kWrite && lane == 0) cnt[i] = 0;
    return;
  }
  const float4 pi = sorted_pos[k];
  int64_t rb, re;
  lane_range(cell_of[i], g, cell_start, lane, rb, re);
  const int len = (int)(re - rb);
  int incl = len;   // inclusive running total over the lanes
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int t = __shfl_up_sync(full, incl, d);
    if (lane >= d) incl += t;
  }
  const int total = __shfl_sync(full, incl, 31);
  const int64_t off = rb - (int64_t)(incl - len);   // candidate number t of range r is atom rb_r + t - excl_r
  // the atom a lane checks in the pass starting at `base` (q < 0: none)
  auto locate = [&](int base) -> int64_t {
    const int kk = base + lane;
    int lo = 0;
#pragma unroll
    for (int step = 16; step >= 1; step >>= 1) {
      const int v = __shfl_sync(full, incl, lo + step - 1);
      if (v <= kk) lo += step;
    }
    const int64_t o = __shfl_sync(full, off, lo);
    return kk < total ? o + kk : -1;
  };
  int64_t w = kWrite ? row_ptr[i] : 0;
  int count = 0;
  int64_t qn = locate(0);
  int jn = -1;
  float4 pn = pi;
  if (qn >= 0) { jn = sorted_idx[qn]; pn = sorted_pos[qn]; }
  for (int base = 0; base < total; base += 32) {
    const int j = jn;
    const float4 pj = pn;
    const bool valid = qn >= 0;
    if (base + 32 < total) {   // warp-uniform
      qn = locate(base + 32);
      if (qn >= 0) { jn = sorted_idx[qn]; pn = sorted_pos[qn]; }
    } else {
      qn = -1;
    }
    const bool hit = valid && (j != i || self_loops) && pair_within(pi, pj, g);
    const unsigned m = __ballot_sync(full, hit);
    if (kWrite && hit) {
      const int64_t o = w + __popc(m & ((1u << lane) - 1u));
      if (o < E) tmp_j[o] = (IdxT)j;
      else atomicOr(err, 4);  // buffers shorter than the counted list: drop, flag
    }
    w += __popc(m);
    count += __popc(m);
  }
  if (!kWrite && lane == 0) cnt[i] = count;
}

// Sort each row's targets (written unsorted into the target row), then write
// the source row and the wrapped vectors.  One warp per atom; rows up to
// kNLStage entries are ranked from shared memory, longer rows are sorted in
// place by a warp-cooperative odd-even transposition sort.
constexpr int kNLStage = 512;

template <class IdxT>
__global__ void __launch_bounds__(256) nl_finish_kernel(int64_t N, NLGeom g, const float* __restrict__ pos,
                                                        const int64_t* __restrict__ row_ptr,
                                                        IdxT* __restrict__ ei_src, IdxT* __restrict__ ei_dst,
                                                        float* __restrict__ vec, int64_t E) {
  __shared__ IdxT stage[8][kNLStage];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = (int64_t)blockIdx.x * 8 + w;
  if (i >= N) return;
  const int64_t b = row_ptr[i], d = row_ptr[i + 1] - b;
  if (d == 0 || b + d > E) return;  // rows past a short E were dropped (flagged by the write pass)
  IdxT* row = ei_dst + b;
  if (d <= kNLStage) {
    for (int64_t k = lane; k < d; k += 32) stage[w][k] = row[k];
    __syncwarp();
    for (int64_t k = lane; k < d; k += 32) {
      const IdxT j = stage[w][k];
      int64_t rank = 0;
      for (int64_t q = 0; q < d; ++q) rank += (stage[w][q] < j);
      row[rank] = j;
    }
  } else {
    for (int64_t phase = 0; phase < d; ++phase) {
      for (int64_t k = 2 * lane + (phase & 1); k + 1 < d; k += 64) {
        IdxT a = row[k], c = row[k + 1];
        if (a > c) { row[k] = c; row[k + 1] = a; }
      }
      __syncwarp();
    }
  }
  __syncwarp();
  const float px = pos[3 * i], py = pos[3 * i + 1], pz = pos[3 * i + 2];
  for (int64_t k = lane; k < d; k += 32) {
    const int64_t j = (int64_t)row[k];
    const int64_t o = b + k;
    ei_src[o] = (IdxT)i;
    if (g.tri) {
      float dx = __fsub_rn(pos[3 * j], px), dy = __fsub_rn(pos[3 * j + 1], py), dz = __fsub_rn(pos[3 * j + 2], pz);
      min_image_tri(dx, dy, dz, g);
      vec[3 * o] = dx;
      vec[3 * o + 1] = dy;
      vec[3 * o + 2] = dz;
    } else {
      vec[3 * o] = min_image(__fsub_rn(pos[3 * j], px), g.L[0]);
      vec[3 * o + 1] = min_image(__fsub_rn(pos[3 * j + 1], py), g.L[1]);
      vec[3 * o + 2] = min_image(__fsub_rn(pos[3 * j + 2], pz), g.L[2]);
    }
  }
}

struct NLWork {
  int* cell_of; int* slot_of; int* cell_cnt; int* cnt;
  int64_t* cell_start; int64_t* scan_tmp;
  int* sorted_idx; float4* sorted_pos;
  size_t bytes;
};

static size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

static NLWork nl_layout(void* base, int64_t N, const NLGeom& g) {
  NLWork w{};
  char* p = static_cast<char*>(base);
  size_t off = 0;
  auto take = [&](size_t b) { char* r = p ? p + off : nullptr; off += align256(b); return r; };
  const int64_t nc = g.ncell;
  w.cell_of = (int*)take(sizeof(int) * N);
  w.slot_of = (int*)take(sizeof(int) * N);
  w.cell_cnt = (int*)take(sizeof(int) * (nc + 1));
  w.cnt = (int*)take(sizeof(int) * (N + 1));
  w.cell_start = (int64_t*)take(sizeof(int64_t) * (nc + 1));
  int64_t st = (int64_t)scan_tmp_elems(nc > N ? nc : N);
  w.scan_tmp = (int64_t*)take(sizeof(int64_t) * st);
  w.sorted_idx = (int*)take(sizeof(int) * N);
  w.sorted_pos = (float4*)take(sizeof(float4) * N);
  w.bytes = off;
  return w;
}

static int nl_prepare(const float* pos, int64_t N, const NLGeom& g, NLWork& w, cudaStream_t st) {
  cudaMemsetAsync(w.cell_cnt, 0, sizeof(int) * (g.ncell + 1), st);
  nl_bin_kernel<<<grid_for(N, 256), 256, 0, st>>>(pos, N, g, w.cell_of, w.slot_of, w.cell_cnt);
  int rc = check_launch("neighbor_list(bin)");
  if (rc) return rc;
  if ((rc = exclusive_scan_i32_to_i64(w.cell_cnt, w.cell_start, g.ncell, w.scan_tmp, st))) return rc;
  nl_scatter_kernel<<<grid_for(N, 256), 256, 0, st>>>(pos, N, w.cell_of, w.slot_of, w.cell_start, w.sorted_idx,
                                                      w.sorted_pos);
  return check_launch("neighbor_list(scatter)");
}

}  // namespace bm

using namespace bm;

extern "C" {

size_t bm_nl_workspace_bytes(int64_t N, const float* box, double cutoff) {
  NLGeom g;
  if (nl_geom(box, cutoff, g)) return 0;
  return nl_layout(nullptr, N, g).bytes;
}

int bm_nl_count(const float* pos, int64_t N, const float* box, double cutoff, bool self_loops, int64_t* row_ptr,
                void* ws, size_t ws_bytes, void* stream) {
  return bm_nl_count_rows(pos, N, N, box, cutoff, self_loops, row_ptr, ws, ws_bytes, stream);
}

int bm_nl_fill(const float* pos, int64_t N, const float* box, double cutoff, bool self_loops, const int64_t* row_ptr,
               int64_t E, int64_t* edge_index, float* vec, void* ws, size_t ws_bytes, void* stream) {
  return bm_nl_fill_rows(pos, N, N, box, cutoff, self_loops, row_ptr, E, edge_index, vec, ws, ws_bytes, stream);
}

}  // extern "C"

namespace bm {

static int nl_count_impl(const float* pos, int64_t N, int64_t n_rows, NLGeom& g, bool self_loops, int64_t* row_ptr,
                         void* ws, size_t ws_bytes, void* stream) {
  BM_REQUIRE(N >= 0 && N < (int64_t(1) << 31), "neighbor_list: bad atom count");
  BM_REQUIRE(row_ptr, "neighbor_list: null row_ptr");
  BM_REQUIRE(n_rows >= 0 && n_rows <= N, "neighbor_list: n_rows must be in [0, N]");
  int rc;
  g.n_rows = n_rows;
  cudaStream_t st = as_stream(stream);
  if (N == 0) {
    cudaMemsetAsync(row_ptr, 0, sizeof(int64_t), st);
    return check_launch("neighbor_list(empty)", 0);
  }
  BM_REQUIRE(pos, "neighbor_list: null positions");
  NLWork w = nl_layout(ws, N, g);
  if (!ws || ws_bytes < w.bytes) return set_error(BM_ERR_WORKSPACE, "neighbor_list: workspace too small");
  if ((rc = nl_prepare(pos, N, g, w, st))) return rc;
  nl_pairs_kernel<false, int64_t><<<grid_for(N * 32, 128), 128, 0, st>>>(N, g, self_loops, w.cell_of, w.cell_start,
                                                             w.sorted_idx, w.sorted_pos, w.cnt, nullptr, nullptr,
                                                             0, nullptr);
  if ((rc = check_launch("neighbor_list(count)"))) return rc;
  return exclusive_scan_i32_to_i64(w.cnt, row_ptr, N, w.scan_tmp, st);
}

}  // namespace bm

extern "C" {

int bm_nl_count_rows(const float* pos, int64_t N, int64_t n_rows, const float* box, double cutoff, bool self_loops,
                     int64_t* row_ptr, void* ws, size_t ws_bytes, void* stream) {
  NLGeom g;
  const int rc = nl_geom(box, cutoff, g);
  return rc ? rc : nl_count_impl(pos, N, n_rows, g, self_loops, row_ptr, ws, ws_bytes, stream);
}

}  // extern "C"

namespace bm {

// Write pass + sort for an already counted list (row_ptr from the count pass,
// cell arrays still valid in the workspace).  E = row_ptr[N].
template <class IdxT>
static int nl_fill_impl(const float* pos, int64_t N, const NLGeom& g, bool self_loops, const int64_t* row_ptr,
                        IdxT* ei_src, IdxT* ei_dst, float* vec, int64_t E, const NLWork& w, cudaStream_t st) {
  int* err = tc::error_flag();
  if (!err) return set_error(BM_ERR_CUDA, "neighbor_list: device error flag unavailable");
  nl_pairs_kernel<true, IdxT><<<grid_for(N * 32, 128), 128, 0, st>>>(N, g, self_loops, w.cell_of, w.cell_start,
                                                                  w.sorted_idx, w.sorted_pos, nullptr, row_ptr,
                                                                  ei_dst, E, err);
  int rc = check_launch("neighbor_list(write)");
  if (rc) return rc;
  nl_finish_kernel<IdxT><<<grid_for(N, 8), 256, 0, st>>>(N, g, pos, row_ptr, ei_src, ei_dst, vec, E);
  return check_launch("neighbor_list(sort)");
}

}  // namespace bm

extern "C" {

}  // extern "C"

namespace bm {

static int nl_fill_rows_impl(const float* pos, int64_t N, int64_t n_rows, NLGeom& g, bool self_loops,
                             const int64_t* row_ptr, int64_t E, int64_t* edge_index, float* vec, void* ws,
                             size_t ws_bytes, void* stream) {
  BM_REQUIRE(N >= 0, "neighbor_list: bad atom count");
  if (N == 0 || E == 0) return BM_OK;
  BM_REQUIRE(n_rows >= 0 && n_rows <= N, "neighbor_list: n_rows must be in [0, N]");
  g.n_rows = n_rows;
  BM_REQUIRE(pos && row_ptr && edge_index && vec, "neighbor_list: null pointer");
  NLWork w = nl_layout(ws, N, g);
  if (!ws || ws_bytes < w.bytes) return set_error(BM_ERR_WORKSPACE, "neighbor_list: workspace too small");
  BM_REQUIRE(E >= 0, "neighbor_list: negative edge count");
  cudaStream_t st = as_stream(stream);
  if (E == 0) return BM_OK;
  return nl_fill_impl<int64_t>(pos, N, g, self_loops, row_ptr, edge_index, edge_index + E, vec, E, w, st);
}

}  // namespace bm

extern "C" {

int bm_nl_fill_rows(const float* pos, int64_t N, int64_t n_rows, const float* box, double cutoff, bool self_loops,
                    const int64_t* row_ptr, int64_t E, int64_t* edge_index, float* vec, void* ws, size_t ws_bytes,
                    void* stream) {
  NLGeom g;
  const int rc = nl_geom(box, cutoff, g);
  return rc ? rc : nl_fill_rows_impl(pos, N, n_rows, g, self_loops, row_ptr, E, edge_index, vec, ws, ws_bytes, stream);
}

size_t bm_nl_workspace_bytes_cell(int64_t N, const float* cell, double cutoff) {
  NLGeom g;
  if (nl_geom_cell(cell, cutoff, g)) return 0;
  return nl_layout(nullptr, N, g).bytes;
}

int bm_nl_count_cell(const float* pos, int64_t N, int64_t n_rows, const float* cell, double cutoff, bool self_loops,
                     int64_t* row_ptr, void* ws, size_t ws_bytes, void* stream) {
  NLGeom g;
  const int rc = nl_geom_cell(cell, cutoff, g);
  return rc ? rc : nl_count_impl(pos, N, n_rows, g, self_loops, row_ptr, ws, ws_bytes, stream);
}

int bm_nl_fill_cell(const float* pos, int64_t N, int64_t n_rows, const float* cell, double cutoff, bool self_loops,
                    const int64_t* row_ptr, int64_t E, int64_t* edge_index, float* vec, void* ws, size_t ws_bytes,
                    void* stream) {
  NLGeom g;
  const int rc = nl_geom_cell(cell, cutoff, g);
  return rc ? rc : nl_fill_rows_impl(pos, N, n_rows, g, self_loops, row_ptr, E, edge_index, vec, ws, ws_bytes, stream);
}

int neighbor_list_cuda(const float* positions, const float* cell, int64_t N, float cutoff, bool self_loops,
                       NeighborListResult* result, void* stream) {
  if (!result) return set_error(BM_ERR_INVALID_ARG, "neighbor_list_cuda: null result");
  result->num_edges = 0;
  result->edge_index = result->d_edge_index = nullptr;
  result->edge_vectors = result->d_edge_vectors = nullptr;
  if (N == 0) return BM_OK;
  cudaStream_t st = as_stream(stream);
  float h_cell[9];
  cudaError_t ce = cudaMemcpyAsync(h_cell, cell, sizeof(h_cell), cudaMemcpyDeviceToHost, st);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
  if (ce != cudaSuccess) return set_error(BM_ERR_CUDA, "neighbor_list_cuda: %s", cudaGetErrorString(ce));
  const float box[3] = {h_cell[0], h_cell[4], h_cell[8]};
  NLGeom g;
  int rc = nl_geom(box, (double)cutoff, g);
  if (rc) return rc;
  NLWork w = nl_layout(nullptr, N, g);
  void* ws = nullptr;
  int64_t* row_ptr = nullptr;
  if ((ce = cudaMalloc(&ws, w.bytes)) != cudaSuccess ||
      (ce = cudaMalloc((void**)&row_ptr, sizeof(int64_t) * (N + 1))) != cudaSuccess) {
    cudaFree(ws);
    return set_error(BM_ERR_CUDA, "neighbor_list_cuda: %s", cudaGetErrorString(ce));
  }
  w = nl_layout(ws, N, g);
  int64_t E = 0;
  rc = bm_nl_count(positions, N, box, (double)cutoff, self_loops, row_ptr, ws, w.bytes, stream);
  if (!rc) {
    ce = cudaMemcpyAsync(&E, row_ptr + N, sizeof(int64_t), cudaMemcpyDeviceToHost, st);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
    if (ce != cudaSuccess) rc = set_error(BM_ERR_CUDA, "neighbor_list_cuda: %s", cudaGetErrorString(ce));
  }
  if (!rc && E > 0) {
    int* ei = nullptr;
    float* vec = nullptr;
    if ((ce = cudaMalloc((void**)&ei, sizeof(int) * 2 * E)) != cudaSuccess ||
        (ce = cudaMalloc((void**)&vec, sizeof(float) * 3 * E)) != cudaSuccess) {
      cudaFree(ei);
      rc = set_error(BM_ERR_CUDA, "neighbor_list_cuda: %s", cudaGetErrorString(ce));
    } else {
      rc = nl_fill_impl<int>(positions, N, g, self_loops, row_ptr, ei, ei + E, vec, E, w, st);
      if (!rc) {
        ce = cudaStreamSynchronize(st);
        if (ce != cudaSuccess) rc = set_error(BM_ERR_CUDA, "neighbor_list_cuda: %s", cudaGetErrorString(ce));
      }
      if (rc) { cudaFree(ei); cudaFree(vec); }
      else {
        result->d_edge_index = result->edge_index = ei;
        result->d_edge_vectors = result->edge_vectors = vec;
        result->num_edges = E;
      }
    }
  }
  cudaStreamSynchronize(st);
  cudaFree(ws);
  cudaFree(row_ptr);
  return rc;
}

void neighbor_list_free(NeighborListResult* r) {
  if (!r) return;
  if (r->d_edge_index) cudaFree(r->d_edge_index);
  if (r->d_edge_vectors) cudaFree(r->d_edge_vectors);
  r->d_edge_index = r->edge_index = nullptr;
  r->d_edge_vectors = r->edge_vectors = nullptr;
  r->num_edges = 0;
}

size_t neighbor_list_estimate_memory(int64_t N, float density, float cutoff) {
  const double per_atom = density * 4.0 / 3.0 * 3.141592653589793 * (double)cutoff * cutoff * cutoff + 1.0;
  return (size_t)((double)N * per_atom * (2 * sizeof(int) + 3 * sizeof(float))) + (size_t)N * sizeof(int) * 4;
}

}  // extern "C"
