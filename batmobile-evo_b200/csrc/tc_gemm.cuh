// tcgen05 (5th-gen tensor core) TF32 GEMM for the per-path channel mixes.
//
//   D[M x N] = sum_k A(m, k) * B(n, k)      (fp32 in, fp32 accumulate in TMEM)
//
// A persistent kernel (one CTA per SM) walks 128 x BN output tiles.  Producer
// warps stream K-slabs of 32 elements through registers into a ring of
// shared-memory stages in the canonical SWIZZLE_128B layouts (K-major: 8-row x
// 128-byte atoms; MN-major tf32: 4 K-rows x 32 MN-element atoms), one thread
// issues tcgen05.mma (kind::tf32, M=128, N=BN, K=8) into one of two TMEM
// accumulators, tcgen05.commit arrives on mbarriers that release ring slots and
// hand finished accumulators to the epilogue warps, which read TMEM with
// tcgen05.ld (one row per thread) while the next tile accumulates.
//
// Accuracy: kind::tf32 reads the top 19 bits of each fp32 operand.  With
// kSplit3 the staged value v (read as hi = its tf32 truncation) gets a second
// tile lo = v - trunc_tf32(v), and D accumulates hi*hi + hi*lo + lo*hi (the
// 3xTF32 scheme): fp32-level results (~1e-6 relative).  Single-pass mode is plain
// TF32 (~5e-4 relative).
//
// Every wait is bounded (~1 s of %globaltimer): on timeout the kernel records an
// error flag (bm_device_error_check), frees TMEM and returns.
#pragma once

#include <cuda.h>
#include <string.h>

#include "bm_common.cuh"

namespace bm {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the completion of phase `parity`; false (and *err set) on
// timeout.  The clock is read once every 1024 polls (about a second in total).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = 0;
#pragma unroll 1
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023) == 0) {
      const uint64_t now = global_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > 1000000000ull) {
        if (err) atomicOr(err, 1);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Whole warp: allocate `ncols` TMEM columns (power of two >= 32); base written to *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Shared-memory matrix descriptor: K-major, SWIZZLE_128B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;  // stride byte offset: next 8 rows
  d |= (uint64_t)1 << 46;             // descriptor version (sm100)
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// MN-major 32-bit operands (tf32) use the SWIZZLE_128B_BASE32B layout: atoms of
// 4 K-rows x 32 MN-elements (4 x 128 B), 32-byte chunks XOR-swizzled with the
// K-row (Swizzle<2,5,2>); `lbo` = bytes between MN blocks of 32, `sbo` = bytes
// between K blocks of 4.
__device__ __forceinline__ uint64_t sdesc_mn_sw128b32(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)1 << 61;  // SWIZZLE_128B_BASE32B
  return d;
}

// Instruction descriptor: kind::tf32, fp32 accumulate; a_mn / b_mn select MN-major operands.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; thread i of the warp gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

constexpr int kBM = 128, kBK = 32;

#ifdef BM_DIAG
static __device__ unsigned long long g_gdiag[16];
#define GD_DECL unsigned long long gd[16] = {0}; unsigned long long gt0 = clock64(), gts = gt0;
#define GD_MARK() gt0 = clock64();
#define GD_ADD(slot) { unsigned long long _n = clock64(); gd[slot] += _n - gt0; gt0 = _n; }
#define GD_FLUSH(tslot) if (lane == 0) { gd[tslot] = clock64() - gts; for (int _i = 0; _i < 16; ++_i) atomicAdd(&g_gdiag[_i], gd[_i]); }
#else
#define GD_DECL
#define GD_MARK()
#define GD_ADD(slot)
#define GD_FLUSH(tslot)
#endif

// --------------------------------------------------------------------------
// Persistent, warp-specialised kernel.  Roles (320 threads):
//   warp 0      TMA: one lane waits for a free ring slot, arms full[slot] with
//               the slab's byte count and issues the 2D tensor copies of the A
//               and B slabs (hardware swizzle, zero fill past the edges);
//   warps 1-4   split (kSplit3 only): wait full[slot]; each thread moves
//               one A row into TMEM (raw value = tf32 hi part, and lo = v -
//               trunc_tf32(v), 32 columns each), writes lo for B into shared
//               memory beside B, fences, arrives on ready[slot];
//   warp 5      MMA: one lane waits ready[slot] (full[slot] in single-pass
//               mode), issues tcgen05.mma (3xTF32: A from TMEM, B from shared
//               memory; single pass: both from shared memory) into one of two
//               TMEM accumulators,
//               commits to empty[slot] and, after a tile's last slab, to
//               tfull[acc];
//   warps 6-9   epilogue: wait tfull[acc], tcgen05.ld their 32 TMEM lanes,
//               store the rows straight to global memory, arrive tempty[acc].
// Tiles (group, M tile, N tile, K split) are dealt round-robin to the CTAs,
// heaviest group first.
//
// Shared-memory operand layouts (per stage, R rows of the operand):
//   K-major : SWIZZLE_128B, 8-row x 128-byte atoms, one TMA box {32 k, R rows};
//   MN-major: SWIZZLE_128B_BASE32B atoms of 4 K-rows x 32 MN-elements (512 B,
//             32-byte chunks XOR-ed with the K-row); each block of 32 MN-elements
//             holds its 32 K-rows contiguously (4 KB, one TMA box {32 mn, 32 k}),
//             so LBO (MN-block stride) = 4096 and SBO (K-block stride) = 512.
// --------------------------------------------------------------------------
constexpr int kSplitWarps = 4, kEpi = 128;
constexpr int kWsThreads = 32 + 32 * kSplitWarps + 32 + kEpi;
constexpr int kMmaWarp = 1 + kSplitWarps;
constexpr int kMaxStages = 8;
#ifndef BM_GEMM_AHI_TMEM
#define BM_GEMM_AHI_TMEM 0
#endif
// TMEM columns per stage for the split A operand: lo only (hi = the raw slab
// in shared memory, which kind::tf32 reads as tf32), or hi and lo.
constexpr int kALoCols = BM_GEMM_AHI_TMEM ? 64 : 32;

template <int BN, bool kSplit3, bool kTmaStore = false>
struct Smem {
  // stage: A (TMA) | B (TMA) | B lo (kSplit3, written by the split warps)
  static constexpr int kA = kBM * 128;
  static constexpr int kB = BN * 128;
  static constexpr int kStage = kA + (kSplit3 ? 2 : 1) * kB;
  // TMA-store epilogue: one 128-row x 32-column staging tile after the ring
  static constexpr int kEpiStage = kTmaStore ? kBM * 128 : 0;
  static constexpr int kBudget = 216 * 1024 - kEpiStage;
  static constexpr int kFit = kBudget / kStage;
  // kSplit3 with BN = 64 fuses two of the three products into one N = 128 MMA
  // (A_hi x [B_hi | B_lo]) and accumulates A_lo x B_hi into its second half, so
  // an accumulator is 2 BN columns wide; the epilogue adds the two halves.
  static constexpr bool kFuse = kSplit3 && BN == 64;
  static constexpr int kAccCols = kFuse ? 2 * BN : BN;
  // kSplit3: TMEM holds 2 accumulators + per stage the A lo part (32 columns;
  // the A hi products read the raw slab from shared memory)
  static constexpr int kTmemFit = kSplit3 ? (512 - 2 * kAccCols) / kALoCols : kMaxStages;
  static constexpr int kFit2 = kFit < kTmemFit ? kFit : kTmemFit;
  static constexpr int kStages = kFit2 > kMaxStages ? kMaxStages : kFit2;
  static constexpr int kBytes = kStages * kStage + kEpiStage + 1024;  // + alignment slack
  static constexpr int kTmemCols = kSplit3 ? 512 : (2 * BN < 32 ? 32 : 2 * BN);
};

// Global view of one GEMM operand: `outer` rows of `inner` fp32 elements,
// rows `pitch` bytes apart (K-major: rows are M/N, inner is K; MN-major: rows
// are K, inner is M/N).
struct Operand {
  const void* base;
  int64_t inner, outer, pitch;
};

// Encodes a 2D fp32 tensor map with box {box_inner, box_outer}; swizzle 0 =
// 128B (K-major atoms), 1 = 128B with 32-byte atoms (MN-major tf32), 2 = 64B
// (16-byte chunk c of 64-byte row r lands at chunk c ^ ((r >> 1) & 3)).
int encode_tmap(CUtensorMap* map, const Operand& op, int box_inner, int box_outer, int swizzle);

// Up to four problems of the same shape family (one per l-group) in one launch.
template <class P>
struct Grouped {
  CUtensorMap ta[4], tb[4], td[4];  // td: output maps of kTmaStore problems
  P p[4];
  int64_t kchunk[4];
  int tiles_m[4], tiles_n[4];
  int start[5];   // tile offsets per group (each tile counted once per K split)
  int ng;
  int splits;
  int total;
};

struct TileInfo {
  int g;
  int64_t m0, n0, kbeg, kend;
  int nk;
};

template <class P, int BN>
__device__ __forceinline__ TileInfo tile_info(const Grouped<P>& G, int id) {
  TileInfo ti;
  const int z = id % G.splits;
  const int rest = id / G.splits;
  int g = 0;
  while (g + 1 < G.ng && rest >= G.start[g + 1]) ++g;
  const int local = rest - G.start[g];
  ti.g = g;
  ti.m0 = (int64_t)(local / G.tiles_n[g]) * kBM;
  ti.n0 = (int64_t)(local % G.tiles_n[g]) * BN;
  const P& p = G.p[g];
  ti.kbeg = (int64_t)z * G.kchunk[g];
  ti.kend = imin64(p.depth(), ti.kbeg + G.kchunk[g]);
  ti.nk = ti.kend > ti.kbeg ? (int)((ti.kend - ti.kbeg + kBK - 1) / kBK) : 0;
  return ti;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// 2D tiled TMA load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 1D bulk copy (no multicast) of `bytes` (multiple of 16, both addresses
// 16-byte aligned) from global to shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// 2D tiled TMA store (bulk group) from shared memory; completion via the bulk-group counters.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Loads one operand slab: R rows (MN) x 32 K starting at (mn0, k0).
template <int R, bool kMN>
__device__ __forceinline__ void tma_slab(uint32_t dst, const CUtensorMap* map, int64_t mn0, int64_t k0, uint64_t* bar) {
  if (!kMN) {
    tma_load_2d(dst, map, (int)k0, (int)mn0, bar);
  } else {
#pragma unroll
    for (int j = 0; j < R / 32; ++j) tma_load_2d(dst + j * 4096, map, (int)(mn0 + 32 * j), (int)k0, bar);
  }
}

template <int R, bool kMN>
__device__ __forceinline__ uint64_t op_desc(uint32_t base, int kk) {
  return kMN ? sdesc_mn_sw128b32(base + kk * 1024, 4096, 512) : sdesc_k_sw128(base + kk * 32);
}

__device__ __forceinline__ float tf32_lo(float v) { return v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

// The 32 K-values of A row `r` from a staged slab.  K-major (SWIZZLE_128B):
// row r at r * 128, 16-byte chunk c at ((c ^ r) & 7) * 16.  MN-major
// (SWIZZLE_128B_BASE32B, 4 KB per block of 32 rows): element (r, k) at
// (r / 32) * 4096 + (k / 4) * 512 + (k % 4) * 128 + ((((r % 32) / 8) ^ (k % 4)) * 32) + (r % 8) * 4.
template <bool kMN>
__device__ __forceinline__ void load_a_row(const uint8_t* st, int r, float (&v)[32]) {
  if (!kMN) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 q = *reinterpret_cast<const float4*>(st + r * 128 + (((c ^ r) & 7) << 4));
      v[4 * c] = q.x; v[4 * c + 1] = q.y; v[4 * c + 2] = q.z; v[4 * c + 3] = q.w;
    }
  } else {
    const uint8_t* blk = st + (r >> 5) * 4096 + (r & 7) * 4;
    const int q = (r >> 3) & 3;
#pragma unroll
    for (int k = 0; k < 32; ++k)
      v[k] = *reinterpret_cast<const float*>(blk + (k >> 2) * 512 + (k & 3) * 128 + ((q ^ (k & 3)) << 5));
  }
}

// Whole warp: 32 consecutive columns of this warp's 32 TMEM lanes (one row per thread).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D (+)= A * B with A read from TMEM (128 lanes = rows, 8 columns = K) and B from shared memory.
__device__ __forceinline__ void mma_tf32_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Problem interface:
//   static constexpr bool kAMN, kBMN          operand rows are MN-contiguous (else K-contiguous)
//   static constexpr const char* kName        launch-site name for the profiler
//   Operand a_op() const, b_op() const        global views of A and B (host)
//   __device__ void store16(int64_t m, int64_t n0, const float (&v)[16], int nvalid, int split)
//                                             row m, columns n0 .. n0+nvalid-1 (n0 % 16 == 0)
//   __host__ __device__ int64_t rows(), cols(), depth()
// Operand bases and pitches are 16-byte aligned; elements past the logical
// end inside a row are zero (padding) or past the tensor map's extent.
template <class P, int BN, bool kSplit3>
__global__ void __launch_bounds__(kWsThreads, 1) tc_gemm_kernel(const __grid_constant__ Grouped<P> G, int* err) {
  using L = Smem<BN, kSplit3, P::kTmaStore>;
  constexpr int S = L::kStages;
  constexpr uint32_t kTx = L::kA + L::kB;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[kMaxStages], ready[kMaxStages], empty[kMaxStages], tfull[2], tempty[2];
  __shared__ uint32_t tmem_base_sh;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;

  if (warp == kMmaWarp) tmem_alloc(&tmem_base_sh, L::kTmemCols);
  if (t == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], kSplitWarps);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) { mbar_init(&tfull[b], 1); mbar_init(&tempty[b], kEpi / 32); }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  bool ok = true;

  if (warp == 0) {
    // ----------------------------------------------------------------- TMA
    int slab = 0;
    GD_DECL
    if (lane == 0) {
      for (int id = blockIdx.x; id < G.total && ok; id += gridDim.x) {
        const TileInfo ti = tile_info<P, BN>(G, id);
        const CUtensorMap* ma = &G.ta[ti.g];
        const CUtensorMap* mb = &G.tb[ti.g];
        for (int kb = 0; kb < ti.nk && ok; ++kb, ++slab) {
          const int s = slab % S;
          GD_ADD(1)
          if (slab >= S) ok = mbar_wait(&empty[s], ((slab / S) - 1) & 1, err);
          GD_ADD(0)
          if (!ok) break;
          const uint32_t st = sbase + s * L::kStage;
          const int64_t k0 = ti.kbeg + (int64_t)kb * kBK;
          mbar_expect_tx(&full[s], kTx);
          tma_slab<kBM, P::kAMN>(st, ma, ti.m0, k0, &full[s]);
          tma_slab<BN, P::kBMN>(st + L::kA, mb, ti.n0, k0, &full[s]);
        }
      }
      // copies still in flight land before the CTA may exit (bounded)
      for (int j = slab - S > 0 ? slab - S : 0; j < slab; ++j) mbar_wait(&full[j % S], (j / S) & 1, nullptr);
      GD_ADD(1)
    }
    GD_FLUSH(15)
    __syncwarp();
  } else if (warp <= kSplitWarps) {
    // --------------------------------------------------------------- split
    if (kSplit3) {
      // thread <-> A row (TMEM lane) 32 * (warp % 4) + lane
      const int quarter = warp & 3;
      const int row = quarter * 32 + lane;
      const int st_t = t - 32;  // 0..127 over the B split
      int slab = 0;
      GD_DECL
      for (int id = blockIdx.x; id < G.total && ok; id += gridDim.x) {
        const TileInfo ti = tile_info<P, BN>(G, id);
        for (int kb = 0; kb < ti.nk && ok; ++kb, ++slab) {
          const int s = slab % S;
          GD_ADD(3)
          ok = mbar_wait(&full[s], (slab / S) & 1, err);
          GD_ADD(2)
          if (!ok) break;
          const uint8_t* st = smem + s * L::kStage;
          float v[32];
          load_a_row<P::kAMN>(st, row, v);
          const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(2 * L::kAccCols + s * kALoCols);
#if BM_GEMM_AHI_TMEM
          tmem_st32(ta, v);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = tf32_lo(v[j]);
          tmem_st32(ta + 32, v);
#else
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = tf32_lo(v[j]);
          tmem_st32(ta, v);
#endif
          uint8_t* sb = smem + s * L::kStage + L::kA;
#pragma unroll 4
          for (int o = st_t * 16; o < L::kB; o += 32 * kSplitWarps * 16) {
            const float4 w = *reinterpret_cast<const float4*>(sb + o);
            *reinterpret_cast<float4*>(sb + L::kB + o) = make_float4(tf32_lo(w.x), tf32_lo(w.y), tf32_lo(w.z), tf32_lo(w.w));
          }
          tmem_wait_st();
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ready[s]);
        }
      }
      GD_ADD(3)
      if (warp == 1) { GD_FLUSH(14) }
    }
  } else if (warp == kMmaWarp) {
    // ----------------------------------------------------------------- MMA
    constexpr uint32_t idesc = idesc_tf32(kBM, BN, P::kAMN ? 1 : 0, P::kBMN ? 1 : 0);
    constexpr uint32_t idesc_t = idesc_tf32(kBM, BN, 0, P::kBMN ? 1 : 0);  // A from TMEM (lane = row)
    int slab = 0, tcount = 0;
    GD_DECL
    for (int id = blockIdx.x; id < G.total && ok; id += gridDim.x, ++tcount) {
      const TileInfo ti = tile_info<P, BN>(G, id);
      const int ab = tcount & 1;
      GD_ADD(6)
      if (tcount >= 2) ok = mbar_wait(&tempty[ab], ((tcount >> 1) - 1) & 1, err) && ok;
      GD_ADD(7)
      tc_fence_after();
      const uint32_t dacc = tmem + (uint32_t)(ab * L::kAccCols);
      for (int kb = 0; kb < ti.nk && ok; ++kb, ++slab) {
        const int s = slab % S;
        GD_ADD(6)
        ok = mbar_wait(kSplit3 ? &ready[s] : &full[s], (slab / S) & 1, err) && ok;
        GD_ADD(4)
        tc_fence_after();
        if (lane == 0 && ok) {
          const uint32_t a_sm = sbase + s * L::kStage, b_hi = a_sm + L::kA, b_lo = b_hi + L::kB;
          const uint32_t a_tm = tmem + (uint32_t)(2 * L::kAccCols + s * kALoCols);
          constexpr uint32_t kLo = BM_GEMM_AHI_TMEM ? 32 : 0;   // A lo column offset in the stage
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk) {
            const uint64_t bd = op_desc<BN, P::kBMN>(b_hi, kk);
#if BM_GEMM_AHI_TMEM
            if constexpr (L::kFuse) {
              // B lo sits right after B hi: one N = 2 BN operand [B_hi | B_lo]
              constexpr uint32_t idesc_f = idesc_tf32(kBM, 2 * BN, 0, P::kBMN ? 1 : 0);
              mma_tf32_ta(dacc, a_tm + kk * 8, bd, idesc_f, (kb > 0 || kk > 0) ? 1u : 0u);
              mma_tf32_ta(dacc + BN, a_tm + kLo + kk * 8, bd, idesc_t, 1u);
            } else if (kSplit3) {
              mma_tf32_ta(dacc, a_tm + kk * 8, bd, idesc_t, (kb > 0 || kk > 0) ? 1u : 0u);
              mma_tf32_ta(dacc, a_tm + kk * 8, op_desc<BN, P::kBMN>(b_lo, kk), idesc_t, 1u);
              mma_tf32_ta(dacc, a_tm + kLo + kk * 8, bd, idesc_t, 1u);
            } else {
#else
            if constexpr (L::kFuse) {
              // B lo sits right after B hi: one N = 2 BN operand [B_hi | B_lo], A hi
              // straight from the staged slab
              constexpr uint32_t idesc_f = idesc_tf32(kBM, 2 * BN, P::kAMN ? 1 : 0, P::kBMN ? 1 : 0);
              mma_tf32(dacc, op_desc<kBM, P::kAMN>(a_sm, kk), bd, idesc_f, (kb > 0 || kk > 0) ? 1u : 0u);
              mma_tf32_ta(dacc + BN, a_tm + kLo + kk * 8, bd, idesc_t, 1u);
            } else if (kSplit3) {
              const uint64_t ad = op_desc<kBM, P::kAMN>(a_sm, kk);
              mma_tf32(dacc, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
              mma_tf32(dacc, ad, op_desc<BN, P::kBMN>(b_lo, kk), idesc, 1u);
              mma_tf32_ta(dacc, a_tm + kLo + kk * 8, bd, idesc_t, 1u);
            } else {
#endif
              mma_tf32(dacc, op_desc<kBM, P::kAMN>(a_sm, kk), bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(&empty[s]);
          if (kb + 1 == ti.nk) mma_commit(&tfull[ab]);
        }
        __syncwarp();
      }
      if (ti.nk == 0 && lane == 0) mma_commit(&tfull[ab]);  // nothing issued: signal at once
      __syncwarp();
    }
    GD_ADD(6)
    GD_FLUSH(13)
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int tcount = 0;
    GD_DECL
    for (int id = blockIdx.x; id < G.total && ok; id += gridDim.x, ++tcount) {
      const TileInfo ti = tile_info<P, BN>(G, id);
      const P& p = G.p[ti.g];
      const int ab = tcount & 1;
      GD_ADD(9)
      ok = mbar_wait(&tfull[ab], (tcount >> 1) & 1, err) && ok;
      GD_ADD(8)
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      if constexpr (P::kTmaStore) {
        // 32 columns at a time through a SWIZZLE_128B staging tile and one TMA
        // store (rows / columns past the edge are clipped by the tensor map)
        uint8_t* stg = smem + (size_t)S * L::kStage;
        const int et = t - (kMmaWarp + 1) * 32;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          float v[32];
          if (ti.nk > 0 && ok) {
            const uint32_t tb = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(ab * L::kAccCols + c0);
            tmem_ld16(tb, v);
            tmem_ld16(tb + 16, v + 16);
            if constexpr (L::kFuse) {
              float w[32];
              tmem_ld16(tb + BN, w);
              tmem_ld16(tb + BN + 16, w + 16);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += w[j];
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.0f;
          }
          if (et == 0) bulk_wait_read0();  // the previous store has read the staging tile
          epi_bar();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(stg + row * 128 + ((j ^ (row & 7)) << 4)) =
                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          fence_proxy_async_smem();
          epi_bar();
          if (et == 0 && ti.n0 + c0 < p.cols())
            tma_store_2d(&G.td[ti.g], (int)(ti.n0 + c0), (int)ti.m0, smem_u32(stg));
        }
      } else {
        const int64_t m = ti.m0 + row;
        const int ncols = (int)imin64(BN, p.cols() - ti.n0);
        const int z = id % G.splits;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          if (ti.nk > 0 && ok) {
            const uint32_t tb = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(ab * L::kAccCols + c0);
            tmem_ld16(tb, v);
            if constexpr (L::kFuse) {
              float w[16];
              tmem_ld16(tb + BN, w);
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] += w[j];
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = 0.0f;
          }
          const int nv = ncols - c0 < 16 ? ncols - c0 : 16;
          if (m < p.rows() && nv > 0) p.store16(m, ti.n0 + c0, v, nv, z);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[ab]);  // TMEM buffer free for the tile after next
    }
    GD_ADD(9)
    if (warp == kMmaWarp + 1) { GD_FLUSH(12) }
    if constexpr (P::kTmaStore) {
      if (t == (kMmaWarp + 1) * 32) bulk_wait0();  // stores complete before the CTA exits
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) tmem_dealloc(tmem, L::kTmemCols);
}

int* error_flag();  // device int of the current device (cudaGetSymbolAddress, cached)

template <class P, int BN, bool kSplit3>
int launch_tc(const P* ps_in, int ng, cudaStream_t st, int splits) {
  using L = Smem<BN, kSplit3, P::kTmaStore>;
  // heaviest K first: tiles are dealt round-robin, so long ones start early
  int order[4] = {0, 1, 2, 3};
  for (int i = 1; i < ng; ++i)
    for (int j = i; j > 0 && ps_in[order[j]].depth() > ps_in[order[j - 1]].depth(); --j) {
      const int tmp = order[j]; order[j] = order[j - 1]; order[j - 1] = tmp;
    }
  Grouped<P> G;
  memset(&G, 0, sizeof(G));
  G.ng = ng;
  G.splits = splits;
  int tiles = 0;
  for (int g = 0; g < ng; ++g) {
    const P& pg = ps_in[order[g]];
    G.p[g] = pg;
    const int64_t M = pg.rows(), N = pg.cols(), K = pg.depth();
    int64_t kchunk = (K + splits - 1) / splits;
    kchunk = ((kchunk + kBK - 1) / kBK) * kBK;
    G.kchunk[g] = kchunk > 0 ? kchunk : kBK;
    G.tiles_n[g] = (int)((N + BN - 1) / BN);
    G.tiles_m[g] = (int)((M + kBM - 1) / kBM);
    G.start[g] = tiles;
    if (M > 0 && N > 0 && K > 0) {
      int rc = P::kAMN ? encode_tmap(&G.ta[g], pg.a_op(), 32, 32, 1) : encode_tmap(&G.ta[g], pg.a_op(), 32, kBM, 0);
      if (rc) return rc;
      rc = P::kBMN ? encode_tmap(&G.tb[g], pg.b_op(), 32, 32, 1) : encode_tmap(&G.tb[g], pg.b_op(), 32, BN, 0);
      if (rc) return rc;
      if constexpr (P::kTmaStore) {
        if ((rc = encode_tmap(&G.td[g], pg.d_op(), 32, kBM, 0))) return rc;
      }
    }
    tiles += (M > 0 && N > 0) ? G.tiles_m[g] * G.tiles_n[g] : 0;
  }
  for (int g = ng; g < 5; ++g) G.start[g] = tiles;
  G.total = tiles * splits;
  if (G.total == 0) return BM_OK;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute((const void*)tc_gemm_kernel<P, BN, kSplit3>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes);
    if (e != cudaSuccess) return set_error(BM_ERR_CUDA, "tc_gemm: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  int* err = error_flag();
  if (!err) return set_error(BM_ERR_CUDA, "tc_gemm: device error flag unavailable");
  const int grid = G.total < kNumSMs ? G.total : kNumSMs;
  tc_gemm_kernel<P, BN, kSplit3><<<grid, kWsThreads, L::kBytes, st>>>(G, err);
  return check_launch(P::kName);
}

}  // namespace tc

int mix_precision();

// Runs ng problems (one per l-group) as one launch; BN from the widest.
template <class P>
int run_tc(const P* ps, int ng, cudaStream_t st, int splits = 1) {
  int64_t ncol = 0;
  for (int g = 0; g < ng; ++g) ncol = ps[g].cols() > ncol ? ps[g].cols() : ncol;
  if (ncol == 0) return BM_OK;
  const bool fast = mix_precision() == 1;
  if (ncol <= 64)
    return fast ? tc::launch_tc<P, 64, false>(ps, ng, st, splits) : tc::launch_tc<P, 64, true>(ps, ng, st, splits);
  return fast ? tc::launch_tc<P, 128, false>(ps, ng, st, splits) : tc::launch_tc<P, 128, true>(ps, ng, st, splits);
}

}  // namespace bm
