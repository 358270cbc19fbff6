// Fused SH -> weighted TP -> scatter interaction layer.
//
// Semantics (the reference's unfused chain, benchmarks/benchmark_e2e_mace.py:323-350):
//   out[n, co, mo] = sum_{e: dst(e)=n} sum_p sum_ci W[p,ci,co] sum_{(m1,m2,mo) in p} c x[src(e),ci,m1] Y_e[m2]
// with Y_e = SH_3(v_e / max(|v_e|, 1e-8)).
//
// Because W does not depend on the edge, the sums are reordered:
//   B_n[ci, m1, m2] = sum_{e -> n} x[src(e), ci, m1] Y_e[m2]            (edge loop, 3xTF32 mma.sync)
//   S_n[p, mo, ci]  = sum_{(m1,m2,mo) in p} c B_n[ci, m1, m2]            (CG, shared memory)
//   out[n, co, mo]  = sum_{p, ci} S_n[p, mo, ci] W[p, ci, co]           (grouped GEMM)
// so neither Y_e nor the per-edge messages are ever written to HBM, the scatter
// is a segmented sum over the target-sorted CSR (no atomics, deterministic),
// and the channel mix runs once per atom instead of once per edge.
//
// Backward:
//   dW = sum_n S_n^T G_n                        (split-K GEMM, deterministic sum)
//   dS_n = G_n W^T                              (grouped GEMM)
//   dB_n = CG^T dS_n ; dY_e = sum x[src] dB_n   (target pass, per edge, 3xTF32 mma.sync) -> dv_e
//   dx_s: the same edge-sum/CG/GEMM machinery run over the SOURCE-sorted CSR
//         with G[dst] in place of x and the CG grouped by l1 (no atomics).
#include "mix_gemm.cuh"

namespace bm {

constexpr int kLT = 256;          // threads per layer CTA
constexpr int kChunkC = 64;       // channels per pass (1024 rows of (c, m))
// Edge-summed tile in shared memory: 256 rows (m2 * 16 + m1) of 64 channels at
// a pitch of 66 floats, rows stored in a permuted order that puts (m1 & 3,
// (m2 >> 1) & 3) in the low four bits of the stored row.  The consumers' stores
// of channel pairs (lanes = 4 m1 x 4 m2 pairs per phase) then hit 16 distinct
// 8-byte bank pairs, and the contractors' loads (compile-time rows, lanes = 16
// channel pairs per phase) stay free of conflicts with plain row offsets.
constexpr int kTilePitch = 66;
constexpr size_t kBsBytes = sizeof(float) * 256 * kTilePitch;
__host__ __device__ constexpr int tile_row(int row) {
  return (row & 3) | (((row >> 5) & 3) << 2) | (((row >> 2) & 3) << 4) | (((row >> 4) & 1) << 6) | (row & 128);
}
__host__ __device__ constexpr int tile_addr(int row, int c) { return tile_row(row) * kTilePitch + c; }

__device__ __forceinline__ void cp_async16_zf(float* dst, const float* src, bool valid) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}

// Balanced contraction of the edge-summed tile into slots: warp K of the
// contraction group (32 threads, two adjacent channels 2 cp, 2 cp + 1 each,
// packed fp32x2 FMAs) owns a contiguous quarter of the output slots, about 153
// of the 611 CG entries.
// MODE 0: tile row (m2 * 16 + m1), outputs grouped by l_out (forward slots).
// MODE 1: tile row (m2 * 16 + m_out), outputs grouped by l1 (input-side backward).
template <int MODE, int K>
__device__ __forceinline__ void contract_part(const float* __restrict__ Bs, int cp, float* __restrict__ slots, int64_t N,
                                              int64_t n, int CF) {
  constexpr int R = MODE == 0 ? kCgpLoOuts[K] : kCgpL1Outs[K];
  float2 acc[R];
#pragma unroll
  for (int i = 0; i < R; ++i) acc[i] = make_float2(0.0f, 0.0f);
#define BM_X(j, row, c) ffma2(acc[j], make_float2((c), (c)), *reinterpret_cast<const float2*>(Bs + tile_addr((row), 2 * cp)));
#define BM_Y(j, g, i)                                                                   \
  {                                                                                     \
    constexpr int OFF_ = kGroupSlotOff[g], ROWS_ = (2 * (g) + 1) * kGroupPaths[g];     \
    *reinterpret_cast<float2*>(slots + N * CF * (int64_t)OFF_ + n * (int64_t)(ROWS_ * CF) + (int64_t)(i) * CF) = acc[j]; \
  }
  if constexpr (MODE == 0) {
    if constexpr (K == 0) { BM_CGP_LO_0(BM_X) BM_CGP_LO_OUT_0(BM_Y) }
    if constexpr (K == 1) { BM_CGP_LO_1(BM_X) BM_CGP_LO_OUT_1(BM_Y) }
    if constexpr (K == 2) { BM_CGP_LO_2(BM_X) BM_CGP_LO_OUT_2(BM_Y) }
    if constexpr (K == 3) { BM_CGP_LO_3(BM_X) BM_CGP_LO_OUT_3(BM_Y) }
  } else {
    if constexpr (K == 0) { BM_CGP_L1_0(BM_X) BM_CGP_L1_OUT_0(BM_Y) }
    if constexpr (K == 1) { BM_CGP_L1_1(BM_X) BM_CGP_L1_OUT_1(BM_Y) }
    if constexpr (K == 2) { BM_CGP_L1_2(BM_X) BM_CGP_L1_OUT_2(BM_Y) }
    if constexpr (K == 3) { BM_CGP_L1_3(BM_X) BM_CGP_L1_OUT_3(BM_Y) }
  }
#undef BM_X
#undef BM_Y
}

// Edge-summed outer products F[other(e)] (x) Y_e over each atom's CSR row, then
// CG contraction into the slot array.  Persistent CTAs (one per SM) walk the
// atoms n_k = blockIdx.x + k * gridDim.x; for each atom and each chunk of 64
// channels the atom's edges are cut into batches of kBatch, which flow in
// stream order through a ring of kBufs batch buffers:
//   warps 12-15        (producers) warp w serves the atoms k = w (mod 4), so the
//                      dependent index loads (CSR row, permutation, edge vector,
//                      source) of four atoms are in flight at once; per batch
//                      one lane per edge evaluates Y_e, the warp waits for its
//                      buffer (stream order), writes Y_e and the source index
//                      and starts bulk copies of the sources' F rows (one
//                      contiguous 4 KB row for 64 channels); lane 0 then arms
//                      full[buf] with the batch's byte count;
//   warps 0-7          (consumers) wait once per batch; a batch of 8 edges is
//                      one k-step of the atom's [1024 x 8] x [8 x 16] product
//                      (rows (channel, m1), k = edge, columns m2) on the tensor
//                      cores: warp w owns channels 8w .. 8w+7 as eight 16-row
//                      m-tiles (two channels x 8 m1 each) and both 8-wide m2
//                      tiles, and issues 3xTF32 mma.sync (hi*hi + hi*lo +
//                      lo*hi, fp32 accumulators in registers); the batch is
//                      released (empty[buf]) once its fragments are read.
//                      At the end of an atom they store the accumulators as
//                      channel pairs into the shared-memory tile
//                      (bfull[tile]) and go on with the next atom;
//   warps 8-11         (contractors) contract each finished tile into slots
//                      (balanced partition, two channels per thread) and
//                      release it (bempty[tile]), overlapped with the
//                      consumers' next atom.
// kBatch divides 32 (the producers' edge groups).
#ifndef BM_AGG_MQ
#define BM_AGG_MQ 4
#endif
#ifndef BM_AGG_BATCH
#define BM_AGG_BATCH 8
#endif
// One edge-summed tile and four batch buffers: the contractors finish an
// atom's tile while the consumers run the next atom's batches, so a second
// tile bought little, and its 66 KB as two more batch buffers keep the
// consumers fed (B200, 5000 atoms, C = 64: 172 -> 161 us per launch).
#ifndef BM_AGG_BUFS
#define BM_AGG_BUFS 4
#endif
#ifndef BM_AGG_TILES
#define BM_AGG_TILES 1
#endif
#ifdef BM_LDIAG
static __device__ unsigned long long g_ldiag[16];
#define LD_DECL unsigned long long ld[16] = {0}; unsigned long long lt0 = clock64(), lts = lt0;
#define LD_ADD(slot) { unsigned long long _n = clock64(); ld[slot] += _n - lt0; lt0 = _n; }
#define LD_MARK() lt0 = clock64();
#define LD_FLUSH(tslot) if (MODE == 0 && lane == 0) { ld[tslot] = clock64() - lts; for (int _i = 0; _i < 16; ++_i) if (ld[_i]) atomicAdd(&g_ldiag[_i], ld[_i]); }
#else
#define LD_DECL
#define LD_ADD(slot)
#define LD_MARK()
#define LD_FLUSH(tslot)
#endif
constexpr int kBatch = BM_AGG_BATCH;
constexpr int kBufs = BM_AGG_BUFS;
static_assert(32 % kBatch == 0, "batches must tile the producers' 32-edge groups");
constexpr int kRing = kBatch * kBufs;
constexpr int kProdWarps = 4;
constexpr int kRowBytes = kChunkC * 16 * 4;           // F row of one channel chunk
constexpr int kSlotBytes = kRowBytes + 160;   // row | Y_e | source index | pad (slot pitch = 8 mod 32 words)
constexpr int kContrWarps = 4;
#ifndef BM_AGG_CW
#define BM_AGG_CW 8
#endif
constexpr int kAggCW = BM_AGG_CW;                     // consumer warps
constexpr int kAggCT = 32 * kAggCW;                   // consumer threads
constexpr int kCPW = kChunkC / kAggCW;                // channels per consumer warp
constexpr int kMT = kCPW;                             // its 16-row m-tiles (two channels x 8 m1 each)
static_assert(kMT % BM_AGG_MQ == 0, "m-tile groups must tile the warp's m-tiles");
constexpr int kAggProdWarp0 = kAggCW + kContrWarps;
constexpr int kTiles = BM_AGG_TILES;     // edge-summed tiles handed to the contractors
constexpr size_t kAggSmem = (size_t)kRing * kSlotBytes + kTiles * kBsBytes + 16;
constexpr int kAggThreads = kAggCT + 32 * (kContrWarps + kProdWarps);

// Bounded spin until *turn == want; false (and *err set) after a few seconds.
__device__ __forceinline__ bool wait_turn(const uint32_t* turn, uint32_t want, int* err) {
  uint64_t t0 = 0;
#pragma unroll 1
  for (uint32_t i = 1; *reinterpret_cast<const volatile uint32_t*>(turn) != want; ++i) {
    __nanosleep(64);  // leave the shared-memory pipe to the consumers
    if ((i & 1023) == 0) {
      const uint64_t now = tc::global_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > 1000000000ull) {
        atomicOr(err, 1);
        return false;
      }
    }
  }
  return true;
}

// Batches the stream holds for atom n: one per kBatch edges per channel chunk.
__device__ __forceinline__ uint32_t atom_batches(const int64_t* __restrict__ row_ptr, int64_t n, int64_t N, int chunks) {
  if (n >= N) return 0;
  const int64_t deg = row_ptr[n + 1] - row_ptr[n];
  return (uint32_t)(((deg + kBatch - 1) / kBatch) * chunks);
}

template <int MODE>
__global__ void __launch_bounds__(kAggThreads, 1)
layer_aggregate_kernel(const float* __restrict__ F, int CF, int CPF, const float* __restrict__ vec,
                       const int64_t* __restrict__ other, const int64_t* __restrict__ row_ptr,
                       const int64_t* __restrict__ perm, float* __restrict__ slots, int64_t N, int64_t NF,
                       const float* __restrict__ escale, int* err) {
  extern __shared__ __align__(16) uint8_t agg_smem[];
  uint8_t* ring = agg_smem;
  float* Bs2 = reinterpret_cast<float*>(agg_smem + (size_t)kRing * kSlotBytes);  // kTiles x [256][kTilePitch]
  __shared__ uint64_t full[kBufs], empty[kBufs], bfull[kTiles], bempty[kTiles];
  __shared__ uint32_t turn;  // next batch allowed to take its buffer (stream order)
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  if (t == 0) {
    turn = 0;
    for (int i = 0; i < kBufs; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], kAggCW);
    }
    for (int i = 0; i < kTiles; ++i) {
      tc::mbar_init(&bfull[i], kAggCW);
      tc::mbar_init(&bempty[i], kContrWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // zero the ring once: the row of an invalid source is never copied and is
  // multiplied by Y_e = 0, so it must hold finite values
  for (int i = t; i < (int)(kRing * kSlotBytes / 16); i += blockDim.x)
    reinterpret_cast<float4*>(ring)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  tc::fence_proxy_async_smem();
  __syncthreads();
  bool ok = true;
  const int chunks = (CF + kChunkC - 1) / kChunkC;

  if (warp >= kAggCW && warp < kAggProdWarp0) {
    // ---------------------------------------------------------- contractors
    const int ct = t - kAggCT, cp = ct & 31, part = ct >> 5;
    uint32_t k = 0;
    LD_DECL
    for (int64_t n = blockIdx.x; n < N && ok; n += gridDim.x) {
      for (int c0 = 0; c0 < CF && ok; c0 += kChunkC, ++k) {
        const uint32_t tile = k % kTiles;
        LD_MARK()
        ok = tc::mbar_wait(&bfull[tile], (k / kTiles) & 1, err);
        ok = __all_sync(0xffffffffu, ok);
        LD_ADD(10)
        if (!ok) break;
        const float* Bs = Bs2 + (size_t)tile * 256 * kTilePitch;
        if (c0 + 2 * cp < CPF) {  // padding channels (>= CF) accumulate zeros
          float* base = slots + c0 + 2 * cp;
          switch (part) {
            case 0: contract_part<MODE, 0>(Bs, cp, base, N, n, CPF); break;
            case 1: contract_part<MODE, 1>(Bs, cp, base, N, n, CPF); break;
            case 2: contract_part<MODE, 2>(Bs, cp, base, N, n, CPF); break;
            default: contract_part<MODE, 3>(Bs, cp, base, N, n, CPF); break;
          }
        }
        __syncwarp();
        LD_ADD(11)
        if (lane == 0) tc::mbar_arrive(&bempty[tile]);
      }
    }
    LD_FLUSH(12)
  } else if (warp >= kAggProdWarp0) {
    // ----------------------------------------------------------- producers
    const int pw = warp - kAggProdWarp0;
    const int64_t step = gridDim.x;
    LD_DECL
    // stream position of this warp's first atom: batches of the atoms before it
    uint32_t bi = 0;
    {
      const uint32_t nb = lane < pw ? atom_batches(row_ptr, blockIdx.x + lane * step, N, chunks) : 0u;
      bi = __reduce_add_sync(0xffffffffu, nb);
    }
    for (int64_t n = blockIdx.x + pw * step; n < N && ok; n += kProdWarps * step) {
      const int64_t eb = row_ptr[n], ee = row_ptr[n + 1];
      for (int c0 = 0; c0 < CF && ok; c0 += kChunkC) {
        const uint32_t bytes = (uint32_t)min(kChunkC, CF - c0) * 64u;
        for (int64_t g0 = eb; g0 < ee && ok; g0 += 32) {
          // up to 32 edges: one lane each
          const int gcnt = (int)imin64(32, ee - g0);
          float yv[16];
          int64_t o = -1;
          if (lane < gcnt) {
            const int64_t e = perm ? perm[g0 + lane] : g0 + lane;
            float x = vec[3 * e], y = vec[3 * e + 1], z = vec[3 * e + 2];
            o = other[e];
            o = (o >= 0 && o < NF) ? o : -1;
            unit3(x, y, z);
            sh_eval<3>(x, y, z, yv);
            if (escale) {  // per-edge scale (radial weight channel): Y_e -> s_e Y_e
              const float sc = escale[e];
#pragma unroll
              for (int b = 0; b < 16; ++b) yv[b] *= sc;
            }
          }
          for (int b0 = 0; b0 < gcnt && ok; b0 += kBatch, ++bi) {
            const int cnt = min(kBatch, gcnt - b0);
            const bool act = lane >= b0 && lane < b0 + cnt;
            const uint32_t buf = bi % kBufs;
            // buffers are taken in stream order, so a buffer's empty barrier is
            // never more than one phase behind the batch waiting for it
            LD_ADD(8)
            if (lane == 0) {
              ok = wait_turn(&turn, bi, err);
              LD_ADD(5)
              if (ok && bi >= kBufs) ok = tc::mbar_wait(&empty[buf], ((bi / kBufs) - 1) & 1, err);
              LD_ADD(6)
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            const uint32_t mine = (act && o >= 0) ? bytes : 0u;
            if (act) {
              uint8_t* sp = ring + (size_t)(buf * kBatch + (lane - b0)) * kSlotBytes;
              float4* yd = reinterpret_cast<float4*>(sp + kRowBytes);
#pragma unroll
              for (int b = 0; b < 4; ++b)
                yd[b] = o >= 0 ? make_float4(yv[4 * b], yv[4 * b + 1], yv[4 * b + 2], yv[4 * b + 3])
                               : make_float4(0.f, 0.f, 0.f, 0.f);  // an invalid source adds nothing
              *reinterpret_cast<int64_t*>(sp + kRowBytes + 64) = o;
              if (o >= 0) tc::bulk_g2s(sp, F + (o * CF + c0) * 16, bytes, &full[buf]);
            }
            const uint32_t total = __reduce_add_sync(0xffffffffu, mine);
            __syncwarp();
            // one arrival per batch: releases the Y / index writes of all lanes
            // and registers the bytes the copies will complete
            if (lane == 0) {
              tc::mbar_expect_tx(&full[buf], total);
              *reinterpret_cast<volatile uint32_t*>(&turn) = bi + 1;
            }
            LD_ADD(7)
          }
        }
      }
      // skip the batches of the other producers' atoms up to this warp's next one
      const uint32_t nb =
          (lane >= 1 && lane < kProdWarps) ? atom_batches(row_ptr, n + lane * step, N, chunks) : 0u;
      bi += __reduce_add_sync(0xffffffffu, nb);
    }
    LD_FLUSH(9)
    // every started copy is consumed before the consumers finish, so nothing
    // is in flight once the CTA reaches its final barrier
  } else {
    // ------------------------------------------------------------ consumers
    uint32_t bi = 0, k = 0;
    LD_DECL
    for (int64_t n = blockIdx.x; n < N && ok; n += gridDim.x) {
      const int64_t eb = row_ptr[n], ee = row_ptr[n + 1];
      for (int c0 = 0; c0 < CF && ok; c0 += kChunkC, ++k) {
        // one batch of 8 edges = one k-step of a [1024 x 8] x [8 x 16] product per
        // atom: warp w owns channels 8 w .. 8 w + 7 (one 16-row m-tile each: the
        // channel's 16 m1 rows), both 8-wide m2 n-tiles; 3xTF32 mma.sync
        const int g = lane >> 2, tq = lane & 3;
        const int cvalid = min(kChunkC, CF - c0);  // channels of this chunk
        float acc[kMT][2][4];
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[mt][nt][i] = 0.0f;
        for (int64_t e0 = eb; e0 < ee; e0 += kBatch, ++bi) {
          const int cnt = (int)imin64(kBatch, ee - e0);
          const uint32_t buf = bi % kBufs;
          LD_MARK()
          if (!tc::mbar_wait(&full[buf], (bi / kBufs) & 1, err)) { ok = false; break; }
          LD_ADD(0)
          const float* s0 = reinterpret_cast<const float*>(ring + (size_t)(buf * kBatch + tq) * kSlotBytes);
          const float* s1 = reinterpret_cast<const float*>(ring + (size_t)(buf * kBatch + tq + 4) * kSlotBytes);
          // B = Y (k = edge slot, n = m2); slots past the batch add nothing
          uint32_t bh[2][2], bl[2][2];
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            split_tf32(tq < cnt ? s0[kChunkC * 16 + 8 * nt + g] : 0.0f, bh[nt][0], bl[nt][0]);
            split_tf32(tq + 4 < cnt ? s1[kChunkC * 16 + 8 * nt + g] : 0.0f, bh[nt][1], bl[nt][1]);
          }
          // m-tile mt: rows 0-7 = channel c, rows 8-15 = channel c + 1 (c = 8 w +
          // 2 (mt / 2)), both at m1 = 8 (mt % 2) + row % 8.  All A loads come first
          // (no branches between them and the MMAs); channels past the chunk's
          // last one read as zeros
          float xr[kMT][4];
          const bool fullw = kCPW * warp + kCPW <= cvalid;
#pragma unroll
          for (int mt = 0; mt < kMT; ++mt) {
            const int cc = kCPW * warp + 2 * (mt >> 1);
            const int o = 16 * cc + 8 * (mt & 1) + g;
            const bool v0 = fullw || cc < cvalid, v1 = fullw || cc + 1 < cvalid;
            xr[mt][0] = v0 ? s0[o] : 0.0f;
            xr[mt][1] = v1 ? s0[o + 16] : 0.0f;
            xr[mt][2] = v0 ? s1[o] : 0.0f;
            xr[mt][3] = v1 ? s1[o + 16] : 0.0f;
          }
          // m-tiles in groups of BM_AGG_MQ, the three terms outermost: 2 BM_AGG_MQ
          // independent accumulators between dependent MMAs (mma.sync latency)
#pragma unroll
          for (int mp = 0; mp < kMT; mp += BM_AGG_MQ) {
            uint32_t ah[BM_AGG_MQ][4], al[BM_AGG_MQ][4];
#pragma unroll
            for (int h = 0; h < BM_AGG_MQ; ++h)
#pragma unroll
              for (int i = 0; i < 4; ++i) split_tf32(xr[mp + h][i], ah[h][i], al[h][i]);
#pragma unroll
            for (int h = 0; h < BM_AGG_MQ; ++h)
#pragma unroll
              for (int nt = 0; nt < 2; ++nt) mma_tf32_16x8x8(acc[mp + h][nt], al[h], bh[nt][0], bh[nt][1]);
#pragma unroll
            for (int h = 0; h < BM_AGG_MQ; ++h)
#pragma unroll
              for (int nt = 0; nt < 2; ++nt) mma_tf32_16x8x8(acc[mp + h][nt], ah[h], bl[nt][0], bl[nt][1]);
#pragma unroll
            for (int h = 0; h < BM_AGG_MQ; ++h)
#pragma unroll
              for (int nt = 0; nt < 2; ++nt) mma_tf32_16x8x8(acc[mp + h][nt], ah[h], bh[nt][0], bh[nt][1]);
          }
          __syncwarp();
          LD_ADD(1)
          if (lane == 0) tc::mbar_arrive(&empty[buf]);
        }
        // hand the tile to the contractors (the tile two atoms back is free once they are done with it)
        const uint32_t tile = k % kTiles;
        LD_MARK()
        if (ok && k >= kTiles) ok = tc::mbar_wait(&bempty[tile], ((k - kTiles) / kTiles) & 1, err);
        LD_ADD(2)
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        float* Bs = Bs2 + (size_t)tile * 256 * kTilePitch;
        // tile row (m2 * 16 + m1), column = channel
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const int c = kCPW * warp + 2 * (mt >> 1), m1 = 8 * (mt & 1) + g, m2 = 8 * nt + 2 * tq;
            *reinterpret_cast<float2*>(Bs + tile_addr(m2 * 16 + m1, c)) = make_float2(acc[mt][nt][0], acc[mt][nt][2]);
            *reinterpret_cast<float2*>(Bs + tile_addr((m2 + 1) * 16 + m1, c)) = make_float2(acc[mt][nt][1], acc[mt][nt][3]);
          }
        __syncwarp();
        LD_ADD(3)
        if (lane == 0) tc::mbar_arrive(&bfull[tile]);
      }
    }
    LD_FLUSH(4)
  }
  __syncthreads();
}

// Per-edge tail of the target pass.  dyv = d(out)/d(s_e Y_e); with a per-edge
// scale s_e the scale gradient is sum_m2 Y_e[m2] dyv[m2] and Y_e sees s_e dyv;
// then the SH and normalisation chain rule gives dv_e.
__device__ __forceinline__ void target_edge_epilogue(int64_t e, float vx, float vy, float vz, float sc, float* dyv,
                                                     float* __restrict__ gv, float* __restrict__ gscale) {
  const float r = unit3(vx, vy, vz);
  if (gscale) {
    float y[16];
    sh_eval<3>(vx, vy, vz, y);
    float ds = 0.0f;
#pragma unroll
    for (int m2 = 0; m2 < 16; ++m2) ds = fmaf(y[m2], dyv[m2], ds);
    gscale[e] = ds;
  }
  if (sc != 1.0f) {
#pragma unroll
    for (int m2 = 0; m2 < 16; ++m2) dyv[m2] *= sc;
  }
  if (gv) {
    float gx, gy, gz;
    sh_grad<3>(vx, vy, vz, dyv, gx, gy, gz);
    unit3_backward(vx, vy, vz, r, gx, gy, gz);
    gv[3 * e] = gx;
    gv[3 * e + 1] = gy;
    gv[3 * e + 2] = gz;
  }
}

// ---------------------------------------------------------------------------
// Target-side backward.  One CTA per target atom n; edges in chunks of 32,
// channels in passes of 16:
//   dB_n[c, m1, m2] = sum_{mo} CG(m1, m2, mo) dS_n[p(m1,m2,mo), mo, c]     (per pass, smem)
//   dY_e[m2]        = sum_{c, m1} x[src e, c, m1] dB_n[c, m1, m2]          (register-blocked)
// then the SH and normalisation chain rule gives dv_e.  The dY product is a
// small GEMM [32 edges x 256] x [256 x 16] per pass: warp w owns K rows
// 32w..32w+31, lane (eg, ks) accumulates 4 edges x 16 m2 over 8 of them, and
// the partial sums are reduced once per edge chunk (shuffles, then smem).
// ---------------------------------------------------------------------------
constexpr int kTC = 16;        // channels per pass (256 K rows)
constexpr int kTE = 32;        // edges per chunk
constexpr int kXPitch = 260;   // X_s row pitch (floats)
constexpr int kTBuf = kSlots * kTC + kTE * kXPitch;  // one pass: dS chunk + gathered x rows
constexpr size_t kTargetSmem = sizeof(float) * (2 * kTBuf + 256 * 16);

__device__ __forceinline__ int dbs_off(int k, int q) {  // float offset of dB row k, m2-quad q
  return k * 16 + (((q ^ k ^ (k >> 4)) & 3) << 2);
}

template <int M1>
__device__ __forceinline__ void dB_row(const float* __restrict__ dSs, int cl, float* d) {
#define BM_X(p, m1, m2, mo, c)                                                                      \
  {                                                                                                \
    constexpr int LO_ = kPathLo[p];                                                                \
    constexpr int SLOT_ = kGroupSlotOff[LO_] + ((mo) - LO_ * LO_) * kGroupPaths[LO_] + kPathPosLo[p]; \
    d[m2] = fmaf((c), dSs[SLOT_ * kTC + cl], d[m2]);                                               \
  }
  if constexpr (M1 == 0) { BM_CG_M1_0(BM_X) }
  if constexpr (M1 == 1) { BM_CG_M1_1(BM_X) }
  if constexpr (M1 == 2) { BM_CG_M1_2(BM_X) }
  if constexpr (M1 == 3) { BM_CG_M1_3(BM_X) }
  if constexpr (M1 == 4) { BM_CG_M1_4(BM_X) }
  if constexpr (M1 == 5) { BM_CG_M1_5(BM_X) }
  if constexpr (M1 == 6) { BM_CG_M1_6(BM_X) }
  if constexpr (M1 == 7) { BM_CG_M1_7(BM_X) }
  if constexpr (M1 == 8) { BM_CG_M1_8(BM_X) }
  if constexpr (M1 == 9) { BM_CG_M1_9(BM_X) }
  if constexpr (M1 == 10) { BM_CG_M1_10(BM_X) }
  if constexpr (M1 == 11) { BM_CG_M1_11(BM_X) }
  if constexpr (M1 == 12) { BM_CG_M1_12(BM_X) }
  if constexpr (M1 == 13) { BM_CG_M1_13(BM_X) }
  if constexpr (M1 == 14) { BM_CG_M1_14(BM_X) }
  if constexpr (M1 == 15) { BM_CG_M1_15(BM_X) }
#undef BM_X
}


__global__ void __launch_bounds__(kLT, 2)
layer_target_bwd_kernel(const float* __restrict__ dS, const float* __restrict__ x, int Ci, int CPi,
                        const float* __restrict__ vec, const int64_t* __restrict__ src,
                        const int64_t* __restrict__ row_ptr, const int64_t* __restrict__ perm,
                        float* __restrict__ gv, int64_t N, int64_t NX, const float* __restrict__ escale,
                        float* __restrict__ gscale) {
  extern __shared__ __align__(16) float smem[];
  float* dBs = smem;                       // [256 K rows][16], quad-swizzled
  float* buf0 = dBs + 256 * 16;            // two pass buffers: dS chunk [156][16], x rows [32][kXPitch]
  float* red = buf0;                       // [8 warps][32 edges][16], reuses the buffers after the passes
  __shared__ int64_t Os[kTE];
  __shared__ float dYs[kTE][16];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int eg = lane >> 2, ks = lane & 3;
  const int64_t n = blockIdx.x;
  const int64_t eb = row_ptr[n], ee = row_ptr[n + 1];
  // dS chunk items (slot, channel quad) this thread copies: global base per item
  constexpr int kItems = (kSlots * 4 + kLT - 1) / kLT;
  const float* dsrc[kItems];
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int it = t + kLT * j, sl = it >> 2;
    dsrc[j] = nullptr;
    if (sl < kSlots) {
      int g = 0;
      while (g < 3 && sl >= group_slot_off(g + 1)) ++g;
      const int local = sl - group_slot_off(g);
      dsrc[j] = dS + N * CPi * (int64_t)group_slot_off(g) + (n * (int64_t)((2 * g + 1) * group_paths(g)) + local) * CPi +
                (it & 3) * 4;
    }
  }
  const int npass = (Ci + kTC - 1) / kTC;
  auto issue = [&](int pass) {
    float* bf = buf0 + (pass & 1) * kTBuf;
    float* xs = bf + kSlots * kTC;
    const int c0 = pass * kTC;
#pragma unroll
    for (int i = 0; i < (kTE * 64) / kLT; ++i) {
      const int q = t + kLT * i, e = q >> 6, kc = q & 63;
      const int64_t o = Os[e];
      const bool v = o >= 0 && c0 + (kc >> 2) < Ci;
      cp_async16_zf(xs + e * kXPitch + kc * 4, v ? x + (o * Ci + c0) * 16 + kc * 4 : x, v);
    }
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      const int it = t + kLT * j;
      if (it < kSlots * 4) {
        const bool v = c0 + (it & 3) * 4 < CPi;
        cp_async16_zf(bf + it * 4, v ? dsrc[j] + c0 : dS, v);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int64_t e0 = eb; e0 < ee; e0 += kTE) {
    const int ne = (int)imin64(kTE, ee - e0);
    if (t < kTE) {
      int64_t s = -1;
      if (t < ne) {
        const int64_t e = perm ? perm[e0 + t] : e0 + t;
        s = src[e];
        if (s < 0 || s >= NX) s = -1;
      }
      Os[t] = s;
    }
    float acc[4][16];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int b = 0; b < 16; ++b) acc[j][b] = 0.0f;
    __syncthreads();
    issue(0);
    for (int pass = 0; pass < npass; ++pass) {
      if (pass + 1 < npass) {
        issue(pass + 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      } else {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
      }
      __syncthreads();
      const float* dSs = buf0 + (pass & 1) * kTBuf;
      const float* Xs = dSs + kSlots * kTC;
      {
        const int cl = t & 15, m1 = t >> 4;
        float d[16];
#pragma unroll
        for (int b = 0; b < 16; ++b) d[b] = 0.0f;
        switch (m1) {
          case 0: dB_row<0>(dSs, cl, d); break;
          case 1: dB_row<1>(dSs, cl, d); break;
          case 2: dB_row<2>(dSs, cl, d); break;
          case 3: dB_row<3>(dSs, cl, d); break;
          case 4: dB_row<4>(dSs, cl, d); break;
          case 5: dB_row<5>(dSs, cl, d); break;
          case 6: dB_row<6>(dSs, cl, d); break;
          case 7: dB_row<7>(dSs, cl, d); break;
          case 8: dB_row<8>(dSs, cl, d); break;
          case 9: dB_row<9>(dSs, cl, d); break;
          case 10: dB_row<10>(dSs, cl, d); break;
          case 11: dB_row<11>(dSs, cl, d); break;
          case 12: dB_row<12>(dSs, cl, d); break;
          case 13: dB_row<13>(dSs, cl, d); break;
          case 14: dB_row<14>(dSs, cl, d); break;
          default: dB_row<15>(dSs, cl, d); break;
        }
        const int k = cl * 16 + m1;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<float4*>(dBs + dbs_off(k, q)) = make_float4(d[4 * q], d[4 * q + 1], d[4 * q + 2], d[4 * q + 3]);
      }
      __syncthreads();
#pragma unroll 2
      for (int i = 0; i < 8; ++i) {
        const int k = 32 * w + 4 * i + ks;
        float xv[4], d[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[j] = Xs[(j * 8 + eg) * kXPitch + k];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v4 = *reinterpret_cast<const float4*>(dBs + dbs_off(k, q));
          d[4 * q] = v4.x; d[4 * q + 1] = v4.y; d[4 * q + 2] = v4.z; d[4 * q + 3] = v4.w;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int b = 0; b < 16; ++b) acc[j][b] = fmaf(xv[j], d[b], acc[j][b]);
      }
      __syncthreads();
    }
    // reduce over the 4 K-lanes of each edge group, then over the 8 warps
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int b = 0; b < 16; ++b) {
        acc[j][b] += __shfl_xor_sync(0xffffffffu, acc[j][b], 1);
        acc[j][b] += __shfl_xor_sync(0xffffffffu, acc[j][b], 2);
      }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float4 v4;
      v4.x = ks == 0 ? acc[j][0] : ks == 1 ? acc[j][4] : ks == 2 ? acc[j][8] : acc[j][12];
      v4.y = ks == 0 ? acc[j][1] : ks == 1 ? acc[j][5] : ks == 2 ? acc[j][9] : acc[j][13];
      v4.z = ks == 0 ? acc[j][2] : ks == 1 ? acc[j][6] : ks == 2 ? acc[j][10] : acc[j][14];
      v4.w = ks == 0 ? acc[j][3] : ks == 1 ? acc[j][7] : ks == 2 ? acc[j][11] : acc[j][15];
      *reinterpret_cast<float4*>(red + (w * kTE + j * 8 + eg) * 16 + ks * 4) = v4;
    }
    __syncthreads();
    for (int i = t; i < kTE * 16; i += kLT) {
      float sum = 0.0f;
#pragma unroll
      for (int ww = 0; ww < 8; ++ww) sum += red[ww * kTE * 16 + i];
      dYs[i >> 4][i & 15] = sum;
    }
    __syncthreads();
    if (t < ne) {
      const int64_t e = perm ? perm[e0 + t] : e0 + t;
      float dyv[16];
#pragma unroll
      for (int m2 = 0; m2 < 16; ++m2) dyv[m2] = dYs[t][m2];
      target_edge_epilogue(e, vec[3 * e], vec[3 * e + 1], vec[3 * e + 2], escale ? escale[e] : 1.0f, dyv, gv, gscale);
    }
    __syncthreads();
  }
}

static size_t slots_floats(int64_t N, int C) { return (size_t)N * pitch4(C) * kSlots; }

static int set_smem(const void* fn, size_t bytes) {
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return set_error(BM_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  return BM_OK;
}

// Shared by the target-side kernels below.
constexpr int kTBufs = 3;                                 // batch buffers in the ring
constexpr size_t kTdSBytes = (size_t)kSlots * 64 * 4;     // dS block of one atom (pitch <= 64)

struct TMeta {  // per-slot edge metadata
  int64_t e;
  float vx, vy, vz;
  int valid;
  float sc;  // per-edge scale of Y (1 without one)
};

// Stream bookkeeping of atom n for the target pass: batches and whether the atom is processed.
__device__ __forceinline__ void target_atom_counts(const int64_t* __restrict__ row_ptr, int64_t n, int64_t N,
                                                   uint32_t& nb, uint32_t& na) {
  nb = 0;
  na = 0;
  if (n < N) {
    const int64_t deg = row_ptr[n + 1] - row_ptr[n];
    nb = (uint32_t)((deg + kBatch - 1) / kBatch);
    na = deg > 0 ? 1u : 0u;
  }
}

// dS block in shared memory: [156 slots][64 channels] (compile-time offsets).
template <int Q>
__device__ __forceinline__ void dB_quarter(const float* __restrict__ dSs, int c, float2 (&d)[16][2]) {
  const float* col = dSs + c;
#define BM_X(m1, j, slot, coeff)                                                \
  {                                                                             \
    float& r_ = ((j) & 1) ? d[m1][(j) >> 1].y : d[m1][(j) >> 1].x;              \
    r_ = fmaf((coeff), col[(slot) * 64], r_);                                   \
  }
#define BM_F() asm volatile("" ::: "memory");
  if constexpr (Q == 0) { BM_CG_M2Q_0(BM_X, BM_F) }
  if constexpr (Q == 1) { BM_CG_M2Q_1(BM_X, BM_F) }
  if constexpr (Q == 2) { BM_CG_M2Q_2(BM_X, BM_F) }
  if constexpr (Q == 3) { BM_CG_M2Q_3(BM_X, BM_F) }
#undef BM_X
#undef BM_F
}

// ---------------------------------------------------------------------------
// Target-side backward on warp-level tensor cores (C_in <= 64).  Per target
// atom n the edge gradient is a product with K = 1024 rows (channel, m1):
//   dY^T[m2, e] = sum_K dB_n^T[m2, K] x[src e]^T[K, e],  dB_n = CG^T dS_n,
// i.e. per batch of 8 edges an [16 x 1024] x [1024 x 8] product (mma.sync
// m16n8k8 tf32, M = m2, N = edges, 3xTF32: hi*hi + hi*lo + lo*hi).
// Persistent CTAs (one per SM) walk the atoms n_k = blockIdx.x + k * gridDim.x:
//   warps 16-17 (producers)  as in the SIMT kernel: per atom the dS block by
//                            bulk copies, then its edges in batches of kBatch
//                            (metadata + the source's x row, one bulk copy of
//                            C_in x 64 bytes into a slot padded to 4 mod 32
//                            words, so a fragment load of 8 edges x 4 K hits 32
//                            banks);
//   warps 0-15 (consumers)   per atom they build dB = CG^T dS (warp w: m2
//                            quarter w % 4, 32 channels, m1 half w / 8) into a
//                            [m2][K] tile; every warp w then keeps the A fragments of its
//                            K slice 64 w .. 64 w + 63 (channels 4w .. 4w+3) in
//                            registers, split into tf32 hi/lo (64 registers);
//                            per batch: 8 k-steps of 3 MMAs on the x fragments
//                            (two loads per k-step), the warp's partial
//                            dY^T[16 x 8] into shared memory;
//   warps 18-19 (epilogue)   per batch (one warp per batch parity): adds the 16
//                            K-slice partials and applies the SH and
//                            normalisation chain rule -> dv_e.
// ---------------------------------------------------------------------------
constexpr int kTMCons = 16;                                  // consumer warps (K slices of 64)
constexpr int kTMProd = 2;                                   // producer warps
constexpr int kTMEpi = kTMCons + kTMProd;                    // first epilogue warp
constexpr int kTMThreads = 32 * (kTMCons + kTMProd + 2);     // two epilogue warps (one per batch parity)
constexpr int kTMSlot = 4096 + 16;                           // x row slot (bytes): 4 mod 32 words
constexpr int kTMdBPitch = 1028;                             // dB tile [m2][K] row pitch (floats)
#ifndef BM_TM_RED
#define BM_TM_RED 2
#endif
constexpr int kTMRed = BM_TM_RED;                            // partial buffers (batches in the epilogue)
constexpr int kTMRedPitch = kTMRed == 2 ? 20 : 16;          // 20: conflict-free consumer stores
constexpr int kTMMeta = 2 * kTBufs;                          // batches of edge metadata in flight                              // partials [warp][edge][m2 (+pad)]
constexpr size_t kTMRingBytes = (size_t)kTBufs * kBatch * kTMSlot;
constexpr size_t kTMdBBytes = (size_t)16 * kTMdBPitch * 4;
constexpr size_t kTMRedBytes = (size_t)kTMRed * kTMCons * kBatch * kTMRedPitch * 4;
constexpr size_t kTMSmem = kTMRingBytes + kTdSBytes + kTMdBBytes + kTMRedBytes + 16;
static_assert(kBatch == 8, "one batch is one 8-wide n-tile of edges");

__device__ __forceinline__ void cons16_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kTMCons) : "memory"); }
__device__ __forceinline__ bool cons16_sync_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(32 * kTMCons)
      : "memory");
  return r != 0;
}

// dB tile element (m2, c, m1): row m2 of 1028 floats, channel c at 16 c, the
// four 16-byte m1 chunks of a channel XOR-swizzled by (c >> 1) & 3 (the
// builder's 8-channel phases and the fragment loads are conflict-free).
__device__ __forceinline__ int dbk_off(int m2, int c, int m1) {
  return m2 * kTMdBPitch + c * 16 + 4 * ((m1 >> 2) ^ ((c >> 1) & 3)) + (m1 & 3);
}

// dB[c, m1, m2] for m2 quarter Q and m1 in 8 H .. 8 H + 7 (compile-time filter
// on the CG list of the quarter).
template <int Q, int H>
__device__ __forceinline__ void dB_quarter_half(const float* __restrict__ dSs, int c, float2 (&d)[16][2]) {
  const float* col = dSs + c;
#define BM_X(m1, j, slot, coeff)                                                \
  if ((m1) >= 8 * H && (m1) < 8 * H + 8) {                                      \
    float& r_ = ((j) & 1) ? d[m1][(j) >> 1].y : d[m1][(j) >> 1].x;              \
    r_ = fmaf((coeff), col[(slot) * 64], r_);                                   \
  }
#define BM_F()
  if constexpr (Q == 0) { BM_CG_M2Q_0(BM_X, BM_F) }
  if constexpr (Q == 1) { BM_CG_M2Q_1(BM_X, BM_F) }
  if constexpr (Q == 2) { BM_CG_M2Q_2(BM_X, BM_F) }
  if constexpr (Q == 3) { BM_CG_M2Q_3(BM_X, BM_F) }
#undef BM_X
#undef BM_F
}

// Builds dB for m2 quarter Q and m1 half H (warp-uniform, lane = channel c)
// into the [m2][K] tile.
template <int Q, int H>
__device__ __forceinline__ void target_build_dBk(const float* dSs, float* dBt, int c, bool cv) {
  float2 d[16][2];  // [m1][m2 pair within the quarter]
#pragma unroll
  for (int i = 0; i < 16; ++i) d[i][0] = d[i][1] = make_float2(0.0f, 0.0f);
  if (cv) dB_quarter_half<Q, H>(dSs, c, d);
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int j = 2 * H; j < 2 * H + 2; ++j) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = (m & 1) ? d[4 * j + u][m >> 1].y : d[4 * j + u][m >> 1].x;
      *reinterpret_cast<float4*>(dBt + dbk_off(4 * Q + m, c, 4 * j)) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

__global__ void __launch_bounds__(kTMThreads, 1)
layer_target_mma_kernel(const float* __restrict__ x, const float* __restrict__ dS, int Ci, int CPi,
                        const float* __restrict__ vec, const int64_t* __restrict__ src,
                        const int64_t* __restrict__ row_ptr, const int64_t* __restrict__ perm,
                        float* __restrict__ gv, int64_t N, int64_t NX, const float* __restrict__ escale,
                        float* __restrict__ gscale, int* err) {
  extern __shared__ __align__(16) uint8_t tm_smem[];
  uint8_t* ring = tm_smem;                                                   // [kTBufs * kBatch][kTMSlot]
  float* dSs = reinterpret_cast<float*>(tm_smem + kTMRingBytes);            // [156][64]
  float* dBt = reinterpret_cast<float*>(tm_smem + kTMRingBytes + kTdSBytes);  // [16][kTMdBPitch]
  float* red = reinterpret_cast<float*>(tm_smem + kTMRingBytes + kTdSBytes + kTMdBBytes);  // [kTMRed][16][8][pitch]
  // edge metadata lives in its own ring of 2 kTBufs batches, released by the
  // epilogue (mempty), so an x-row buffer is free as soon as the consumers are done
  __shared__ TMeta meta[kTMMeta * kBatch];
  __shared__ uint64_t full[kTBufs], empty[kTBufs], mempty[kTMMeta], dfull, dempty, red_full[kTMRed], red_empty[kTMRed];
  __shared__ uint32_t turn;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  if (t == 0) {
    turn = 0;
    for (int i = 0; i < kTBufs; ++i) {
      tc::mbar_init(&full[i], 1);
      tc::mbar_init(&empty[i], kTMCons);
    }
    for (int i = 0; i < kTMMeta; ++i) tc::mbar_init(&mempty[i], 1);
    tc::mbar_init(&dfull, 1);
    tc::mbar_init(&dempty, kTMCons);  // every consumer warp builds a part of dB
    for (int i = 0; i < kTMRed; ++i) {
      tc::mbar_init(&red_full[i], kTMCons);
      tc::mbar_init(&red_empty[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // zero the x ring once: bytes past C_in x 64 of a slot are never written, and
  // the fragment loads read all 64 channels (dB is zero there)
  for (int i = t; i < (int)(kTMRingBytes / 16); i += blockDim.x)
    reinterpret_cast<float4*>(ring)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  tc::fence_proxy_async_smem();
  __syncthreads();
  bool ok = true;
  const uint32_t row_bytes = (uint32_t)Ci * 64u;
#ifdef BM_LDIAG
  constexpr int MODE = 0;
#endif
  LD_DECL

  if (warp >= kTMCons && warp < kTMEpi) {
    // ----------------------------------------------------------- producers
    const int pw = warp - kTMCons;
    const int64_t step = gridDim.x;
    uint32_t bi = 0, ac = 0;
    {
      uint32_t nb, na;
      target_atom_counts(row_ptr, blockIdx.x + lane * step, N, nb, na);
      if (lane >= pw) nb = na = 0;
      bi = __reduce_add_sync(0xffffffffu, nb);
      ac = __reduce_add_sync(0xffffffffu, na);
    }
    for (int64_t n = blockIdx.x + pw * step; n < N && ok; n += kTMProd * step) {
      const int64_t eb = row_ptr[n], ee = row_ptr[n + 1];
      if (ee > eb) {
        LD_MARK()
        if (lane == 0) {
          ok = wait_turn(&turn, bi, err);
          if (ok && ac >= 1) ok = tc::mbar_wait(&dempty, (ac - 1) & 1, err);
        }
        LD_ADD(8)
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok) {
          if (CPi == 64) {
            if (lane < 4) {
              const int g = lane;
              const uint32_t rows = (uint32_t)((2 * g + 1) * group_paths(g));
              tc::bulk_g2s(dSs + (size_t)group_slot_off(g) * 64,
                           dS + N * 64 * (int64_t)group_slot_off(g) + n * (int64_t)rows * 64, rows * 256u, &dfull);
            }
          } else {
            for (int sl = lane; sl < kSlots; sl += 32) {
              int g = 0;
              while (g < 3 && sl >= group_slot_off(g + 1)) ++g;
              const int local = sl - group_slot_off(g);
              const int64_t rows = (2 * g + 1) * group_paths(g);
              tc::bulk_g2s(dSs + (size_t)sl * 64, dS + N * CPi * (int64_t)group_slot_off(g) + (n * rows + local) * CPi,
                           (uint32_t)CPi * 4u, &dfull);
            }
          }
          __syncwarp();
          if (lane == 0) tc::mbar_expect_tx(&dfull, (uint32_t)kSlots * (uint32_t)CPi * 4u);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        ++ac;
        for (int64_t g0 = eb; g0 < ee && ok; g0 += 32) {
          const int gcnt = (int)imin64(32, ee - g0);
          TMeta m{};
          int64_t srow = -1;
          if (lane < gcnt) {
            const int64_t e = perm ? perm[g0 + lane] : g0 + lane;
            const int64_t sidx = src[e];
            srow = (sidx >= 0 && sidx < NX) ? sidx : -1;
            m.e = e;
            m.vx = vec[3 * e];
            m.vy = vec[3 * e + 1];
            m.vz = vec[3 * e + 2];
            m.valid = srow >= 0 ? 1 : 0;
            m.sc = escale ? escale[e] : 1.0f;
          }
          for (int b0 = 0; b0 < gcnt && ok; b0 += kBatch, ++bi) {
            const int cnt = min(kBatch, gcnt - b0);
            const bool act = lane >= b0 && lane < b0 + cnt;
            const uint32_t buf = bi % kTBufs;
            LD_MARK()
            const uint32_t mb = bi % kTMMeta;
            if (lane == 0) {
              if (b0 > 0 || g0 > eb) ok = wait_turn(&turn, bi, err);  // the first batch holds the turn already
              if (ok && bi >= kTMMeta) ok = tc::mbar_wait(&mempty[mb], ((bi / kTMMeta) - 1) & 1, err);
              if (ok && bi >= kTBufs) ok = tc::mbar_wait(&empty[buf], ((bi / kTBufs) - 1) & 1, err);
            }
            LD_ADD(9)
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            const uint32_t mine = (act && srow >= 0) ? row_bytes : 0u;
            if (act) {
              const int sl = buf * kBatch + (lane - b0);
              meta[mb * kBatch + (lane - b0)] = m;
              if (srow >= 0) tc::bulk_g2s(ring + (size_t)sl * kTMSlot, x + srow * (int64_t)Ci * 16, row_bytes, &full[buf]);
            }
            const uint32_t total = __reduce_add_sync(0xffffffffu, mine);
            __syncwarp();
            if (lane == 0) {
              tc::mbar_expect_tx(&full[buf], total);
              *reinterpret_cast<volatile uint32_t*>(&turn) = bi + 1;
            }
          }
        }
      }
      uint32_t nb = 0, na = 0;
      if (lane >= 1 && lane < kTMProd) target_atom_counts(row_ptr, n + lane * step, N, nb, na);
      bi += __reduce_add_sync(0xffffffffu, nb);
      ac += __reduce_add_sync(0xffffffffu, na);
    }
    LD_FLUSH(10)
  } else if (warp >= kTMEpi) {
    // ------------------------------------------------------------ epilogue
    // warp kTMEpi + p takes the batches of parity p: dY_e = sum of the 16 K-slice
    // partials, then the SH and normalisation chain rule -> dv_e; lane = (edge
    // lane / 4, m2 quarter lane % 4)
    const int je = lane >> 2, mq = lane & 3;
    const uint32_t mine = (uint32_t)(warp - kTMEpi);
    uint32_t bi = 0;
    for (int64_t n = blockIdx.x; n < N && ok; n += gridDim.x) {
      const int64_t eb = row_ptr[n], ee = row_ptr[n + 1];
      for (int64_t e0 = eb; e0 < ee && ok; e0 += kBatch, ++bi) {
        const int cnt = (int)imin64(kBatch, ee - e0);
        const uint32_t par = bi & 1, rb = bi % kTMRed;
        if (par != mine) continue;
        LD_MARK()
        if (!tc::mbar_wait(&red_full[rb], (bi / kTMRed) & 1, err)) { ok = false; break; }
        LD_ADD(11)
        const float* rp = red + (size_t)rb * kTMCons * kBatch * kTMRedPitch + je * kTMRedPitch + 4 * mq;
        float4 dq = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kTMCons; ++w) {
          const float4 r4 = *reinterpret_cast<const float4*>(rp + w * kBatch * kTMRedPitch);
          dq.x += r4.x; dq.y += r4.y; dq.z += r4.z; dq.w += r4.w;
        }
        // the partials are in registers: hand the buffer back before the chain rule
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&red_empty[rb]);
        float dyv[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int srcl = (lane & ~3) + k;
          dyv[4 * k] = __shfl_sync(0xffffffffu, dq.x, srcl);
          dyv[4 * k + 1] = __shfl_sync(0xffffffffu, dq.y, srcl);
          dyv[4 * k + 2] = __shfl_sync(0xffffffffu, dq.z, srcl);
          dyv[4 * k + 3] = __shfl_sync(0xffffffffu, dq.w, srcl);
        }
        if (mq == 0 && je < cnt) {
          const TMeta mm = meta[(bi % kTMMeta) * kBatch + je];
          if (!mm.valid) {  // the ring slot of an invalid source holds stale rows
#pragma unroll
            for (int m2 = 0; m2 < 16; ++m2) dyv[m2] = 0.0f;
          }
          target_edge_epilogue(mm.e, mm.vx, mm.vy, mm.vz, mm.sc, dyv, gv, gscale);
        }
        __syncwarp();
        LD_ADD(12)
        if (lane == 0) tc::mbar_arrive(&mempty[bi % kTMMeta]);
      }
    }
    LD_FLUSH(13)
  } else {
    // ----------------------------------------------------------- consumers
    const int g = lane >> 2, tq = lane & 3;
    uint32_t bi = 0, ac = 0;
    bool stuck = false;  // a bounded wait of this warp gave up in the edge loop (warp-uniform)
    for (int64_t n = blockIdx.x; n < N && ok; n += gridDim.x) {
      const int64_t eb = row_ptr[n], ee = row_ptr[n + 1];
      if (ee <= eb) continue;
      LD_MARK()
      const bool gave_up = stuck || !__all_sync(0xffffffffu, tc::mbar_wait(&dfull, ac & 1, err));
      ++ac;
      // every warp is done with the previous atom's tile; if any consumer gave
      // up on a wait, all consumer warps leave here together
      if (cons16_sync_or(gave_up)) { ok = false; break; }
      LD_ADD(0)
      {
        // warp w builds m2 quarter w % 4, channels 32 ((w / 4) % 2) + lane, m1 half w / 8
        const int cb = ((warp >> 2) & 1) * 32 + lane;
        const bool cbv = cb < Ci;
        switch (warp & 3) {
          case 0: if (warp < 8) target_build_dBk<0, 0>(dSs, dBt, cb, cbv); else target_build_dBk<0, 1>(dSs, dBt, cb, cbv); break;
          case 1: if (warp < 8) target_build_dBk<1, 0>(dSs, dBt, cb, cbv); else target_build_dBk<1, 1>(dSs, dBt, cb, cbv); break;
          case 2: if (warp < 8) target_build_dBk<2, 0>(dSs, dBt, cb, cbv); else target_build_dBk<2, 1>(dSs, dBt, cb, cbv); break;
          default: if (warp < 8) target_build_dBk<3, 0>(dSs, dBt, cb, cbv); else target_build_dBk<3, 1>(dSs, dBt, cb, cbv); break;
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&dempty);
      }
      LD_ADD(1)
      cons16_sync();
      LD_ADD(2)
      // A fragments of this warp's K slice: k-step s covers channel 4 w + s / 2,
      // m1 = 8 (s % 2) + 0..7; a0 = dB^T[g][t], a1 = [g+8][t], a2 = [g][t+4], a3 = [g+8][t+4]
      uint32_t ah[8][4], al[8][4];
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const int c = 4 * warp + (s >> 1), m1 = 8 * (s & 1) + tq;
        split_tf32(dBt[dbk_off(g, c, m1)], ah[s][0], al[s][0]);
        split_tf32(dBt[dbk_off(g + 8, c, m1)], ah[s][1], al[s][1]);
        split_tf32(dBt[dbk_off(g, c, m1 + 4)], ah[s][2], al[s][2]);
        split_tf32(dBt[dbk_off(g + 8, c, m1 + 4)], ah[s][3], al[s][3]);
      }
      LD_ADD(3)
      for (int64_t e0 = eb; e0 < ee && !stuck; e0 += kBatch, ++bi) {
        const uint32_t buf = bi % kTBufs, rb = bi % kTMRed;
        LD_MARK()
        // warp votes: the warp stays converged and meets the others at the next cons16_sync_or
        if (!__all_sync(0xffffffffu, tc::mbar_wait(&full[buf], (bi / kTBufs) & 1, err))) { stuck = true; break; }
        LD_ADD(4)
        // red[rb] is free once the epilogue has finished the batch kTMRed back
        if (bi >= kTMRed && !__all_sync(0xffffffffu, tc::mbar_wait(&red_empty[rb], ((bi / kTMRed) - 1) & 1, err))) {
          stuck = true;
          break;
        }
        LD_ADD(5)
        // B fragments: b0 = x[src of slot g][K0 + t], b1 = [K0 + t + 4]; slots past
        // the batch hold finite stale rows whose results the epilogue drops
        const float* xs = reinterpret_cast<const float*>(ring + (size_t)(buf * kBatch + g) * kTMSlot) + 64 * warp + tq;
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          uint32_t bh0, bl0, bh1, bl1;
          split_tf32(xs[8 * s], bh0, bl0);
          split_tf32(xs[8 * s + 4], bh1, bl1);
          mma_tf32_16x8x8(acc[s & 1], al[s], bh0, bh1);
          mma_tf32_16x8x8(acc[s & 1], ah[s], bl0, bl1);
          mma_tf32_16x8x8(acc[s & 1], ah[s], bh0, bh1);
        }
        // partial dY^T: d0 = (m2 g, edge 2t), d1 = (g, 2t+1), d2 = (g+8, 2t), d3 = (g+8, 2t+1)
        float* rp = red + ((size_t)rb * kTMCons + warp) * kBatch * kTMRedPitch;
        rp[(2 * tq) * kTMRedPitch + g] = acc[0][0] + acc[1][0];
        rp[(2 * tq + 1) * kTMRedPitch + g] = acc[0][1] + acc[1][1];
        rp[(2 * tq) * kTMRedPitch + g + 8] = acc[0][2] + acc[1][2];
        rp[(2 * tq + 1) * kTMRedPitch + g + 8] = acc[0][3] + acc[1][3];
        __syncwarp();
        LD_ADD(6)
        if (lane == 0) {
          tc::mbar_arrive(&empty[buf]);
          tc::mbar_arrive(&red_full[rb]);
        }
      }
    }
    LD_FLUSH(7)
  }
  __syncthreads();
}

template <int MODE>
static int launch_aggregate(const float* F, int CF, const float* vec, const int64_t* other, const int64_t* row_ptr,
                            const int64_t* perm, float* slots, int64_t N, int64_t NF, const float* escale,
                            cudaStream_t st) {
  int rc = set_smem((const void*)layer_aggregate_kernel<MODE>, kAggSmem);
  if (rc) return rc;
  int* err = tc::error_flag();
  if (!err) return set_error(BM_ERR_CUDA, "layer aggregate: device error flag unavailable");
  const unsigned grid = (unsigned)imin64(N, kNumSMs);
  layer_aggregate_kernel<MODE><<<grid, kAggThreads, kAggSmem, st>>>(F, CF, pitch4(CF), vec, other, row_ptr, perm,
                                                                    slots, N, NF, escale, err);
  return check_launch(MODE == 0 ? "layer_fwd(aggregate)" : "layer_bwd(source aggregate)");
}

}  // namespace bm

using namespace bm;

extern "C" {

size_t bm_layer_fwd_workspace_bytes(int64_t N, int64_t, int Ci, int Co) {
  return (slots_floats(N, Ci) + (size_t)pack_floats(kPackFwd, Ci, Co)) * sizeof(float);
}

int bm_layer_fwd(const float* x, const float* v, const float* W, const int64_t* src, const int64_t* row_ptr_dst,
                 const int64_t* perm_dst, float* out, float* slots_out, int64_t N, int64_t E, int Ci, int Co,
                 void* ws, size_t ws_bytes, void* stream) {
  return bm_layer_fwd_scaled(x, v, W, src, row_ptr_dst, perm_dst, nullptr, out, slots_out, N, E, Ci, Co, ws, ws_bytes,
                             stream);
}

int bm_layer_fwd_scaled(const float* x, const float* v, const float* W, const int64_t* src,
                        const int64_t* row_ptr_dst, const int64_t* perm_dst, const float* edge_scale, float* out,
                        float* slots_out, int64_t N, int64_t E, int Ci, int Co, void* ws, size_t ws_bytes,
                        void* stream) {
  return bm_layer_fwd_targets(x, v, W, src, row_ptr_dst, perm_dst, edge_scale, out, slots_out, N, N, E, Ci, Co, ws,
                              ws_bytes, stream);
}

int bm_layer_fwd_targets(const float* x, const float* v, const float* W, const int64_t* src,
                         const int64_t* row_ptr_dst, const int64_t* perm_dst, const float* edge_scale, float* out,
                         float* slots_out, int64_t N, int64_t NS, int64_t E, int Ci, int Co, void* ws,
                         size_t ws_bytes, void* stream) {
  BM_REQUIRE(N >= 0 && NS >= N && E >= 0 && Ci > 0 && Co > 0, "layer_fwd: bad sizes");
  if (N == 0) return BM_OK;
  BM_REQUIRE(N < (int64_t(1) << 31), "layer_fwd: too many atoms");
  BM_REQUIRE(x && W && out && row_ptr_dst && (E == 0 || (v && src)), "layer_fwd: null pointer");
  if (!ws || ws_bytes < bm_layer_fwd_workspace_bytes(N, E, Ci, Co))
    return set_error(BM_ERR_WORKSPACE, "layer_fwd: workspace too small");
  float* S = slots_out ? slots_out : static_cast<float*>(ws);
  float* Wf = static_cast<float*>(ws) + slots_floats(N, Ci);
  cudaStream_t st = as_stream(stream);
  const int CPi = pitch4(Ci);
  int rc = pack_weights(W, Ci, Co, kPackFwd, Wf, st);
  if (rc) return rc;
  if ((rc = launch_aggregate<0>(x, Ci, v, src, row_ptr_dst, perm_dst, S, N, NS, edge_scale, st))) return rc;
  MixOut ps[4];
  for (int g = 0; g < 4; ++g)
    ps[g] = MixOut{S + slot_group_offset(g, N, CPi), N * (2 * g + 1), (int64_t)kGroupPaths[g] * CPi,
             Wf + pack_group_offset(kPackFwd, g, Ci, Co), Co, out, 2 * g + 1, g * g};
  if ((rc = run_mix4(ps, st))) return rc;
  return BM_OK;
}

size_t bm_layer_bwd_workspace_bytes(int64_t N, int64_t E, int Ci, int Co) {
  return bm_layer_bwd_targets_workspace_bytes(N, N, E, Ci, Co);
}

size_t bm_layer_bwd_targets_workspace_bytes(int64_t N, int64_t NS, int64_t, int Ci, int Co) {
  size_t f = slots_floats(N, Ci) + slots_floats(NS, Co) + (size_t)N * 16 * pitch4(Co) +
             (size_t)pack_floats(kPackDs, Ci, Co) + (size_t)pack_floats(kPackDx, Ci, Co) +
             (size_t)kMaxSplits * kNumPaths * Ci * Co;
  return f * sizeof(float) + 256;
}

int bm_layer_bwd(const float* x, const float* v, const float* W, const int64_t* src, const int64_t* dst,
                 const int64_t* rpd, const int64_t* pd, const int64_t* rps, const int64_t* ps, const float* S,
                 const float* G, float* gx, float* gv, float* gW, int64_t N, int64_t E, int Ci, int Co, void* ws,
                 size_t ws_bytes, void* stream) {
  return bm_layer_bwd_scaled(x, v, W, src, dst, rpd, pd, rps, ps, nullptr, S, G, gx, gv, gW, nullptr, N, E, Ci, Co, ws,
                             ws_bytes, stream);
}

int bm_layer_bwd_scaled(const float* x, const float* v, const float* W, const int64_t* src, const int64_t* dst,
                        const int64_t* rpd, const int64_t* pd, const int64_t* rps, const int64_t* ps,
                        const float* edge_scale, const float* S, const float* G, float* gx, float* gv, float* gW,
                        float* grad_scale, int64_t N, int64_t E, int Ci, int Co, void* ws, size_t ws_bytes,
                        void* stream) {
  return bm_layer_bwd_targets(x, v, W, src, dst, rpd, pd, rps, ps, edge_scale, S, G, gx, gv, gW, grad_scale, N, N, E,
                              Ci, Co, ws, ws_bytes, stream);
}

int bm_layer_bwd_targets(const float* x, const float* v, const float* W, const int64_t* src, const int64_t* dst,
                         const int64_t* rpd, const int64_t* pd, const int64_t* rps, const int64_t* ps,
                         const float* edge_scale, const float* S, const float* G, float* gx, float* gv, float* gW,
                         float* grad_scale, int64_t N, int64_t NS, int64_t E, int Ci, int Co, void* ws,
                         size_t ws_bytes, void* stream) {
  BM_REQUIRE(N >= 0 && NS >= N && E >= 0 && Ci > 0 && Co > 0, "layer_bwd: bad sizes");
  BM_REQUIRE(!grad_scale || edge_scale, "layer_bwd: grad_scale needs edge_scale");
  cudaStream_t st = as_stream(stream);
  if (N == 0) {
    if (gW) cudaMemsetAsync(gW, 0, sizeof(float) * kNumPaths * Ci * Co, st);
    if (gx && NS > 0) cudaMemsetAsync(gx, 0, sizeof(float) * NS * Ci * 16, st);
    return check_launch("layer_bwd(empty)", 0);
  }
  BM_REQUIRE(x && W && G && S && rpd && rps && (E == 0 || (v && src && dst)), "layer_bwd: null pointer");
  if (!ws || ws_bytes < bm_layer_bwd_targets_workspace_bytes(N, NS, E, Ci, Co))
    return set_error(BM_ERR_WORKSPACE, "layer_bwd: workspace too small");
  const int CPi = pitch4(Ci), CPo = pitch4(Co);
  float* dS = static_cast<float*>(ws);
  float* Es = dS + slots_floats(N, Ci);
  float* Gt = Es + slots_floats(NS, Co);
  float* Ws = Gt + (size_t)N * 16 * CPo;
  float* Wd = Ws + pack_floats(kPackDs, Ci, Co);
  float* part = Wd + pack_floats(kPackDx, Ci, Co);
  int rc;
  const bool edge_pass = (gv || grad_scale) && E > 0;
  if (gW || edge_pass) {
    if ((rc = pack_irreps_groups(G, N, Co, Gt, st))) return rc;
  }
  if (gW) {
    const int64_t stride = (int64_t)kNumPaths * Ci * Co;
    const int splits = dw_splits_all(N, Ci, Co);
    MixWeights ps[4];
    for (int g = 0; g < 4; ++g)
      ps[g] = MixWeights{S + slot_group_offset(g, N, CPi), kGroupPaths[g] * CPi, N * (2 * g + 1),
                   Gt + (size_t)N * g * g * CPo, CPo, Co, lo_group(g), Ci, CPi, part, stride};
    if ((rc = run_mix4(ps, st, splits))) return rc;
    if ((rc = sum_splits(part, stride, splits, gW, stride, st))) return rc;
  }
  if (edge_pass) {
    if ((rc = pack_weights(W, Ci, Co, kPackDs, Ws, st))) return rc;
    MixSlots ps[4];
    for (int g = 0; g < 4; ++g)
      ps[g] = MixSlots{Gt + (size_t)N * g * g * CPo, N * (2 * g + 1), CPo, Ws + pack_group_offset(kPackDs, g, Ci, Co),
                 kGroupPaths[g] * CPi, dS + slot_group_offset(g, N, CPi)};
    if ((rc = run_mix4(ps, st))) return rc;
    if (Ci <= 64) {
      if ((rc = set_smem((const void*)layer_target_mma_kernel, kTMSmem))) return rc;
      int* err = tc::error_flag();
      if (!err) return set_error(BM_ERR_CUDA, "layer_bwd: device error flag unavailable");
      layer_target_mma_kernel<<<(unsigned)imin64(N, kNumSMs), kTMThreads, kTMSmem, st>>>(
          x, dS, Ci, CPi, v, src, rpd, pd, gv, N, NS, edge_scale, grad_scale, err);
    } else {
      if ((rc = set_smem((const void*)layer_target_bwd_kernel, kTargetSmem))) return rc;
      layer_target_bwd_kernel<<<(unsigned)N, kLT, kTargetSmem, st>>>(dS, x, Ci, CPi, v, src, rpd, pd, gv, N, NS,
                                                                       edge_scale, grad_scale);
    }
    if ((rc = check_launch("layer_bwd(target)"))) return rc;
  }
  if (gx) {
    if ((rc = pack_weights(W, Ci, Co, kPackDx, Wd, st))) return rc;
    if ((rc = launch_aggregate<1>(G, Co, v, dst, rps, ps, Es, NS, N, edge_scale, st))) return rc;
    MixOut ps[4];
    for (int g = 0; g < 4; ++g)
      ps[g] = MixOut{Es + slot_group_offset(g, NS, CPo), NS * (2 * g + 1), (int64_t)kGroupPaths[g] * CPo,
               Wd + pack_group_offset(kPackDx, g, Ci, Co), Ci, gx, 2 * g + 1, g * g};
    if ((rc = run_mix4(ps, st))) return rc;
  }
  return BM_OK;
}

}  // extern "C"

#ifdef BM_LDIAG
extern "C" __attribute__((visibility("default"))) int bm_ldiag_read(unsigned long long* out) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(out, bm::g_ldiag, sizeof(unsigned long long) * 16);
  unsigned long long z[16] = {0};
  cudaMemcpyToSymbol(bm::g_ldiag, z, sizeof(z));
  return 0;
}
#endif
#ifdef BM_DIAG
extern "C" __attribute__((visibility("default"))) int bm_gdiag_read(unsigned long long* out) {
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(out, bm::tc::g_gdiag, sizeof(unsigned long long) * 16);
  unsigned long long z[16] = {0};
  cudaMemcpyToSymbol(bm::tc::g_gdiag, z, sizeof(z));
  return 0;
}
#endif
