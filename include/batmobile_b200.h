/*
 * batmobile_b200.h -- C ABI of libbatmobile_b200.so, the sm_100a (B200)
 * implementation of batmobile's equivariant message-passing hot path at
 * L_max = 3: spherical harmonics, the 34-path Clebsch-Gordan tensor product,
 * the fused SH -> TP -> scatter layer and the periodic cell-list neighbour
 * list.
 *
 * Conventions shared by every entry point
 *  - All array arguments are DEVICE pointers to dense row-major data unless a
 *    comment says "host".  float is IEEE fp32, indices are int64 unless noted.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *    Every call is asynchronous with respect to the host unless noted.
 *  - Outputs are caller-owned.  Entry points that need scratch memory take a
 *    (workspace, workspace_bytes) pair sized by the matching *_workspace_bytes
 *    query; none of them allocates device memory, except the reference-
 *    compatible neighbor_list_cuda() which allocates its result exactly as the
 *    reference's does.
 *  - Return value is a bm_status; on failure bm_last_error() gives a message.
 *    No C++ exception crosses this boundary.
 *
 * Each declaration names the reference interface it replaces
 * (paths relative to the batmobile-evo source tree).
 */
#ifndef BATMOBILE_B200_H_
#define BATMOBILE_B200_H_

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  BM_OK = 0,
  BM_ERR_INVALID_ARG = 1,  /* shape/size/pointer check failed               */
  BM_ERR_CUDA = 2,         /* a CUDA launch or runtime call failed          */
  BM_ERR_UNSUPPORTED = 3,  /* e.g. SH backward for L_max > 3 (as reference) */
  BM_ERR_CAPACITY = 4,     /* a documented size limit was exceeded          */
  BM_ERR_WORKSPACE = 5,    /* workspace too small                           */
  BM_ERR_TIMEOUT = 6       /* a bounded device-side wait gave up            */
} bm_status;

const char* bm_status_string(int status);
/* Message of the last failure on the calling host thread. */
const char* bm_last_error(void);
int bm_version(void);
/* Number of kernels this library has launched in the process so far. */
int64_t bm_launch_count(void);
/* Launches `blocks` x 256 threads of `iters` x 8 dependent-chain FMAs
 * (2 * 8 * iters FLOP per thread): a peak-fp32 probe for SIMT rooflines.
 * scratch: one device float (written only in a case that cannot occur). */
int bm_probe_fp32(float* scratch, int iters, int blocks, void* stream);
/* Measurement helper: the warp-level tf32 MMA rate of the device (mma.sync
 * m16n8k8, 8 independent accumulators per warp, `blocks` CTAs of 256 threads,
 * `iters` x 8 MMAs per warp), the denominator for the edge-sum and target passes.
 * No reference counterpart (measurement only). */
int bm_probe_mma_tf32(float* scratch, int iters, int blocks, void* stream);
/* Precision of the per-path channel mixes, which run on the tensor cores:
 * 0 (default) = fp32-accurate (TF32 hi/lo split, three passes, ~1e-6 relative);
 * 1 = single-pass TF32 (~5e-4 relative; inside the 2e-3 tolerance allowed for a tf32 mix). */
int bm_set_mix_precision(int mode);
int bm_get_mix_precision(void);
/* Launch profiler.  Between start and stop the library records a CUDA event on
 * `stream` after every kernel it launches (all launches must go to that
 * stream); bm_profile_mark records a boundary (call it before an API call so
 * host time is not charged to its first kernel).  After stop, entry i gives a
 * launch site's name, launch count and total device milliseconds, each launch
 * timed from the previous event to its own. */
int bm_profile_start(void* stream);
int bm_profile_mark(void);
int bm_profile_stop(void);
int bm_profile_count(void);
int bm_profile_entry(int i, char* name, int name_len, int64_t* launches, double* total_ms);
/* Blocks until the current device is idle, reads and clears the device-side
 * error flag: BM_ERR_TIMEOUT if a bounded wait in a pipelined kernel gave up,
 * BM_ERR_CAPACITY if a neighbour-list fill was given fewer edge slots than the
 * list has (the extra edges are dropped, nothing is written past E),
 * BM_ERR_INVALID_ARG if bm_csr_reverse met an edge without its reverse. */
int bm_device_error_check(void);
/* Self-test of the bounded device waits (no counterpart in the reference, which
 * has no bounded waits): one thread waits on an mbarrier that nothing arrives
 * on; the wait gives up after about a second and the kernel returns.  Blocks
 * until done and returns bm_device_error_check(): BM_ERR_TIMEOUT, with the
 * flag cleared and the context usable for the next call. */
int bm_selftest_wait_timeout(void* stream);

/* ---------------------------------------------------------------- paths -- */
/* Replaces batteries::get_num_paths_l3 (src/tensor_product/tensor_product.cu:203). */
int bm_tp_num_paths(void);
/* Host int32 [34*3] (l1, l2, l_out) per path.
 * Replaces batteries::get_path_info_l3 (src/tensor_product/tensor_product.cu:207). */
int bm_tp_path_info(int32_t* out_host);

/* ---------------------------------------------------- spherical harmonics -- */
/* Y[E, (L_max+1)^2] from unit vectors v[E,3]; 0 <= L_max <= 6.
 * Replaces batteries::spherical_harmonics_dispatch
 * (src/spherical_harmonics/spherical_harmonics.cu:296-314). */
int bm_sh_fwd(const float* v, float* Y, int64_t E, int L_max, void* stream);
/* grad_v[E,3] = sum_lm grad_Y[lm] dY_lm/dv (no sphere projection); L_max <= 6
 * (l <= 3 analytic; l = 4..6 by dual numbers through the recurrence -- the
 * reference stops at 3 and returns cudaErrorInvalidValue above).
 * Replaces batteries::spherical_harmonics_backward_dispatch
 * (src/spherical_harmonics/spherical_harmonics_backward.cu:440-463). */
int bm_sh_bwd(const float* v, const float* grad_Y, float* grad_v, int64_t E, int L_max,
              void* stream);

/* ------------------------------------------------- simple tensor product -- */
/* out[N,16] = sum over the 611 CG entries c * a[m1] * b[m2] (all 34 paths, weight 1).
 * Replaces batteries::tensor_product_simple_l3 (src/tensor_product/tensor_product.cu:159-176). */
int bm_tp_simple_fwd(const float* a, const float* b, float* out, int64_t N, void* stream);
/* Replaces batteries::tensor_product_simple_backward_l3
 * (src/tensor_product/tensor_product_backward.cu:1007-1026). */
int bm_tp_simple_bwd(const float* a, const float* b, const float* grad_out, float* grad_a,
                     float* grad_b, int64_t N, void* stream);

/* ----------------------------------------------- weighted tensor product -- */
/* out[N,Co,16] = sum_p sum_ci W[p,ci,Co] * CG_p(x[n,ci,:], Y[n,:]).
 * Replaces batteries::tensor_product_l3 (src/tensor_product/tensor_product.cu:178-201). */
size_t bm_tp_fwd_workspace_bytes(int64_t N, int C_in, int C_out);
int bm_tp_fwd(const float* x, const float* Y, const float* W, float* out, int64_t N, int C_in,
              int C_out, void* workspace, size_t workspace_bytes, void* stream);
/* Any of grad_x / grad_Y / grad_W may be NULL (skipped), as the reference's
 * needs_*_grad flags.  Replaces batteries::tensor_product_backward_l3
 * (src/tensor_product/tensor_product_backward.cu:948-1005). */
size_t bm_tp_bwd_workspace_bytes(int64_t N, int C_in, int C_out);
int bm_tp_bwd(const float* x, const float* Y, const float* W, const float* grad_out,
              float* grad_x, float* grad_Y, float* grad_W, int64_t N, int C_in, int C_out,
              void* workspace, size_t workspace_bytes, void* stream);

/* Same result as bm_tp_fwd, but allocates nothing and takes no workspace: for
 * callers that cannot provide device scratch (an FFI host without a device
 * allocator, or a loop that reserves all device memory up front and must not
 * call cudaMalloc mid-step).  Its scratch is a fixed 24 MiB array inside the
 * library (bm_tp_fwd_noalloc_max_floats() floats), held on every GPU that
 * loads the library until exit; a call whose bm_tp_fwd workspace (about
 * N * C_in * 156 floats plus the repacked weights) exceeds it returns
 * BM_ERR_CAPACITY.  All calls share the array: calls that overlap on the GPU
 * race.  The first call on a device resolves the array's address (make it
 * before any stream capture).  No counterpart in the reference. */
size_t bm_tp_fwd_noalloc_max_floats(void);
int bm_tp_fwd_noalloc(const float* x, const float* Y, const float* W, float* out, int64_t N, int C_in,
                      int C_out, void* stream);

/* --------------------------------------------------------------- graph -- */
/* COO [2,E] (row 0 source, row 1 target) -> CSR by target: row_ptr[N+1],
 * col_idx[E] = original edge ids, ascending inside each row (deterministic).
 * Replaces batteries::edge_index_to_csr (src/message_passing/fused_message_passing.cu:108-165). */
size_t bm_csr_workspace_bytes(int64_t N_atoms, int64_t E);
int bm_edge_index_to_csr(const int64_t* edge_index, int64_t* row_ptr, int64_t* col_idx,
                         int64_t N_atoms, int64_t E, void* workspace, size_t workspace_bytes,
                         void* stream);
/* Reverse-edge index of a SYMMETRIC CSR with sorted rows (a full neighbour
 * list): rev[k] = index of the edge (j, i) for the entry k = (i, j).  rev is the
 * target-grouped permutation of the list (row_ptr serves both orders), i.e. the
 * col_idx bm_edge_index_to_csr returns for the flipped edge index, computed by
 * binary search instead of count + scan + fill + sort.  A missing reverse edge
 * gives -1 and raises the device error flag (bm_device_error_check). */
int bm_csr_reverse(const int64_t* row_ptr, const int64_t* col_idx, int64_t N_atoms, int64_t E,
                   int64_t* rev, void* stream);
/* messages[E,C,16] = TP_simple(x[src[e], c, :], Y(v[e])).  v are unit vectors.
 * Replaces batteries::fused_sh_tp_simple (src/message_passing/fused_sh_tp.cu:125-146). */
int bm_fused_sh_tp_simple(const float* v, const float* x, const int64_t* src, float* messages,
                          int64_t E, int64_t N_atoms, int C, void* stream);
/* out[n,c,:] = sum over CSR row n of TP_simple(x[edge_index[0][e], c], Y(v[e])),
 * e = col_idx[k] (original edge id).  Deterministic segmented sum, no atomics.
 * Replaces batteries::fused_message_passing_simple
 * (src/message_passing/fused_message_passing.cu:257-280). */
int bm_fused_mp_simple(const float* x, const float* v, const int64_t* edge_index,
                       const int64_t* row_ptr, const int64_t* col_idx, float* out,
                       int64_t N_atoms, int64_t E, int C, void* stream);
/* out[n,co,:] = sum over CSR slot k of row n, sum_ci W2[ci,co] *
 * TP_simple(x[col_idx[k], ci], Y(v[k])): col_idx holds SOURCE ATOMS and v is in
 * CSR order -- the contract of the reference binding (python/bindings.cpp:719-737).
 * Replaces batteries::fused_message_passing
 * (src/message_passing/fused_message_passing.cu:376-400). */
size_t bm_fused_mp_weighted_workspace_bytes(int64_t N_atoms, int C_in, int C_out);
int bm_fused_mp_weighted(const float* x, const float* v, const float* W2, const int64_t* row_ptr,
                         const int64_t* col_idx, float* out, int64_t N_atoms, int64_t E,
                         int C_in, int C_out, void* workspace, size_t workspace_bytes,
                         void* stream);

/* --------------------------------------- fused interaction layer --------------- */
/* out[n,co,:] = sum over edges e with dst[e]==n of
 *     sum_p sum_ci W[p,ci,co] * CG_p(x[src[e],ci,:], Y(v[e]/max(|v[e]|,1e-8)))
 * i.e. the reference's unfused chain  normalise -> spherical_harmonics ->
 * x[src] gather -> tensor_product -> scatter_add(dst)
 * (benchmarks/benchmark_e2e_mace.py:323-350; examples/mace_inference.py:134-175)
 * in one pass: messages and Y never reach HBM, the channel mix is applied
 * once per target atom after the segmented edge sum.
 * Target CSR (row_ptr_dst, perm_dst) comes from bm_edge_index_to_csr.
 * slots_out [N * 156 * P] (P = C_in rounded up to a multiple of 4) receives the
 * per-atom CG aggregates the backward pass needs; NULL keeps them in the
 * workspace.  The workspace is always required (it also holds the weights
 * repacked for the tensor-core channel mix). */
size_t bm_layer_fwd_workspace_bytes(int64_t N_atoms, int64_t E, int C_in, int C_out);
int bm_layer_fwd(const float* x, const float* v, const float* W, const int64_t* src,
                 const int64_t* row_ptr_dst, const int64_t* perm_dst, float* out,
                 float* slots_out, int64_t N_atoms, int64_t E, int C_in, int C_out,
                 void* workspace, size_t workspace_bytes, void* stream);
/* Gradients of bm_layer_fwd.  row_ptr_src/perm_src: CSR of the edges by SOURCE
 * (bm_edge_index_to_csr on the flipped edge index).  slots: the forward's
 * slots_out.  grad_x / grad_v / grad_W may each be NULL. */
size_t bm_layer_bwd_workspace_bytes(int64_t N_atoms, int64_t E, int C_in, int C_out);
int bm_layer_bwd(const float* x, const float* v, const float* W, const int64_t* src,
                 const int64_t* dst, const int64_t* row_ptr_dst, const int64_t* perm_dst,
                 const int64_t* row_ptr_src, const int64_t* perm_src, const float* slots,
                 const float* grad_out, float* grad_x, float* grad_v, float* grad_W,
                 int64_t N_atoms, int64_t E, int C_in, int C_out, void* workspace,
                 size_t workspace_bytes, void* stream);
/* Per-edge radial weights: the same pass with Y_e scaled by edge_scale[e]
 * (one radial channel k of W_e = sum_k R_k(e) W_k -- the weight net's last
 * linear layer -- so out = sum_k layer(x, v, W_k, R_k)), and its gradient
 * grad_scale[e] = d(out . grad_out)/d edge_scale[e].  edge_scale may be NULL
 * (all ones); grad_scale may be NULL and needs edge_scale.  The reference's
 * e3nn baseline builds W_e with nn.Linear(1, weight_numel) of the edge length
 * (benchmarks/benchmark_e2e_mace.py:462-497), i.e. K = 2 channels (r, 1). */
int bm_layer_fwd_scaled(const float* x, const float* v, const float* W, const int64_t* src,
                        const int64_t* row_ptr_dst, const int64_t* perm_dst, const float* edge_scale,
                        float* out, float* slots_out, int64_t N_atoms, int64_t E, int C_in, int C_out,
                        void* workspace, size_t workspace_bytes, void* stream);
int bm_layer_bwd_scaled(const float* x, const float* v, const float* W, const int64_t* src,
                        const int64_t* dst, const int64_t* row_ptr_dst, const int64_t* perm_dst,
                        const int64_t* row_ptr_src, const int64_t* perm_src, const float* edge_scale,
                        const float* slots, const float* grad_out, float* grad_x, float* grad_v,
                        float* grad_W, float* grad_scale, int64_t N_atoms, int64_t E, int C_in,
                        int C_out, void* workspace, size_t workspace_bytes, void* stream);
/* Target subset: only the first N_targets atoms are targets (row_ptr_dst has
 * N_targets + 1 entries, out / slots / grad_out have N_targets rows), while
 * sources index all N_sources rows of x (grad_x has N_sources rows).  This is
 * the owned-atoms-first layout of a spatial domain: owned atoms are targets,
 * ghost atoms only sources, so the forward, the slot gradients and the weight
 * gradient skip the ghost rows.  The plain entry points are these with
 * N_targets = N_sources.  The reference has no sharded path; these serve the
 * build's slab decomposition. */
int bm_layer_fwd_targets(const float* x, const float* v, const float* W, const int64_t* src,
                         const int64_t* row_ptr_dst, const int64_t* perm_dst, const float* edge_scale,
                         float* out, float* slots_out, int64_t N_targets, int64_t N_sources, int64_t E,
                         int C_in, int C_out, void* workspace, size_t workspace_bytes, void* stream);
size_t bm_layer_bwd_targets_workspace_bytes(int64_t N_targets, int64_t N_sources, int64_t E, int C_in, int C_out);
int bm_layer_bwd_targets(const float* x, const float* v, const float* W, const int64_t* src,
                         const int64_t* dst, const int64_t* row_ptr_dst, const int64_t* perm_dst,
                         const int64_t* row_ptr_src, const int64_t* perm_src, const float* edge_scale,
                         const float* slots, const float* grad_out, float* grad_x, float* grad_v,
                         float* grad_W, float* grad_scale, int64_t N_targets, int64_t N_sources, int64_t E,
                         int C_in, int C_out, void* workspace, size_t workspace_bytes, void* stream);
/* grad_pos[n] = sum_{e: dst=n} grad_v[e] - sum_{e: src=n} grad_v[e]
 * (v[e] = pos[dst] - pos[src] + periodic shift), deterministic segmented sums.
 * Replaces the torch index_add_ chain the reference relies on for forces
 * (benchmarks/benchmark_e2e_mace.py:412-419, :909). */
int bm_edge_grad_to_pos(const float* grad_v, const int64_t* row_ptr_dst, const int64_t* perm_dst,
                        const int64_t* row_ptr_src, const int64_t* perm_src, float* grad_pos,
                        int64_t N_atoms, void* stream);

/* ------------------------------------------------------- neighbour list -- */
/* Orthorhombic periodic cell list.  Edge set: every ordered pair (i, j), i != j
 * (or i == j too with self_loops), with d = p_i - p_j,
 * d -= rint(d / L) * L (true division, per axis), (dx*dx + dy*dy) + dz*dz <=
 * float(cutoff^2), evaluated in fp32 without contraction -- the predicate of
 * the reference's brute-force check (benchmarks/benchmark_neighbor_list_standalone.py:110-125).
 * Output order: lexicographic (i, j); row 0 = i (source), row 1 = j (target);
 * vec[e] = p_j - p_i min-imaged the same way.  box_host: host float[3] box
 * lengths.  Two calls: bm_nl_count fills row_ptr[N+1] (by source i); the
 * caller reads row_ptr[N] (= E), allocates edge_index[2,E] and vec[E,3], then
 * bm_nl_fill writes the edges.  Both calls must get the same positions and the
 * same workspace (the cell arrays built by the count are reused).  The fill
 * writes at most E edges: if the count it reads holds more, the extra edges
 * are dropped and bm_device_error_check() reports BM_ERR_CAPACITY. */
size_t bm_nl_workspace_bytes(int64_t N, const float* box_host, double cutoff);
int bm_nl_count(const float* pos, int64_t N, const float* box_host, double cutoff, bool self_loops,
                int64_t* row_ptr, void* workspace, size_t workspace_bytes, void* stream);
int bm_nl_fill(const float* pos, int64_t N, const float* box_host, double cutoff, bool self_loops,
               const int64_t* row_ptr, int64_t E, int64_t* edge_index, float* vec, void* workspace,
               size_t workspace_bytes, void* stream);

/* Row-restricted variant for domain decomposition: only atoms i < n_rows get
 * rows (edges (i, j) with i < n_rows, j any of the N atoms).  Because the
 * predicate is symmetric, the rows of the owned atoms of a slab listed first
 * are exactly the incoming edges of those atoms, grouped by target. */
int bm_nl_count_rows(const float* pos, int64_t N, int64_t n_rows, const float* box_host, double cutoff,
                     bool self_loops, int64_t* row_ptr, void* workspace, size_t workspace_bytes, void* stream);
int bm_nl_fill_rows(const float* pos, int64_t N, int64_t n_rows, const float* box_host, double cutoff,
                    bool self_loops, const int64_t* row_ptr, int64_t E, int64_t* edge_index, float* vec,
                    void* workspace, size_t workspace_bytes, void* stream);

/* General periodic cell (triclinic boxes).  `cell_host` is a host float[9],
 * row-major, rows = lattice vectors a, b, c (positions p = s H for fractional
 * s).  The reference reads only the diagonal of its cell
 * (src/neighbor_list/neighbor_list.cu:260-267); these entry points extend the
 * same edge-set contract to any cell: the minimum image is taken in fractional
 * coordinates, s = d Hinv, s -= rint(s), d = s H (row-vector products summed
 * left to right, each operation rounded on its own, Hinv = inverse(H) computed
 * in float64 and rounded to fp32), then (dx*dx + dy*dy) + dz*dz <=
 * float(cutoff^2).  A cell with zero off-diagonal entries gives exactly the
 * orthorhombic result above.  n_rows as in bm_nl_count_rows (N for all rows).
 * Same two-call protocol and workspace rules as bm_nl_count / bm_nl_fill. */
size_t bm_nl_workspace_bytes_cell(int64_t N, const float* cell_host, double cutoff);
int bm_nl_count_cell(const float* pos, int64_t N, int64_t n_rows, const float* cell_host, double cutoff,
                     bool self_loops, int64_t* row_ptr, void* workspace, size_t workspace_bytes, void* stream);
int bm_nl_fill_cell(const float* pos, int64_t N, int64_t n_rows, const float* cell_host, double cutoff,
                    bool self_loops, const int64_t* row_ptr, int64_t E, int64_t* edge_index, float* vec,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Reference-compatible neighbour-list ABI, bound by the reference through
 * ctypes (benchmarks/benchmark_neighbor_list.py:18-47,
 * benchmarks/benchmark_e2e_mace.py:38-61).  Same struct layout and semantics
 * as include/neighbor_list.cuh:25-33 and src/neighbor_list/neighbor_list.cu:455-478:
 * `cell` is a DEVICE float[9] (diagonal used), edge_index is int32 [2,E]
 * (row 0 = i, row 1 = j), edge_vectors [E,3] = p_j - p_i min-imaged; the
 * result owns cudaMalloc'd memory released by neighbor_list_free.  Unlike the
 * reference the edge order is deterministic (lexicographic (i, j)). */
typedef struct {
  int* edge_index;
  float* edge_vectors;
  int64_t num_edges;
  int* d_edge_index;
  float* d_edge_vectors;
} NeighborListResult;
int neighbor_list_cuda(const float* positions, const float* cell, int64_t N, float cutoff,
                       bool self_loops, NeighborListResult* result, void* stream);
void neighbor_list_free(NeighborListResult* result);
size_t neighbor_list_estimate_memory(int64_t N, float density, float cutoff);

#ifdef __cplusplus
}
#endif

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#endif /* BATMOBILE_B200_H_ */
