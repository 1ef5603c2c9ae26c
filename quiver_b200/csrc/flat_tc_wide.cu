// Tensor-core (tcgen05) screen for wide rows and large k: dimensions up to 768 (fp16 operands
// padded to whole 64-column atoms) and best lists of up to 256 groups (k up to 204).
//
// Same arithmetic and certificate as the screen in flat_tc.cu (fp16 MMA with float32
// accumulation in TMEM, 8-row groups, per-query best lists, exact re-rank and certificate in
// flat.cu); what changes is the data movement, which the row width dictates:
//   * one 128-query tile per unit, whose 128 x kpad fp16 operand (up to 192 KB) stays on chip for
//     the whole unit: its first 512 columns in tensor memory (the 256 TMEM columns the two
//     accumulator slots leave free; the epilogue warps store them there with tcgen05.st, and the
//     MMAs read A from TMEM), the rest (columns 512..767) in shared memory. That leaves shared
//     memory to a ring of stages of up to four 64-column K atoms of a row tile (two 64 KB stages
//     at kpad 768), so the issuing thread waits on one barrier per sixteen 128 x 128 x 16 MMAs;
//   * accumulator slots (128 columns each, two of them) are released by their own barrier,
//     because a stage no longer covers a whole row tile;
//   * best lists live in global memory (L2-resident, one region per CTA, entry i of query lane l
//     at i * 128 + l, so a warp's accesses coalesce): 128 queries x up to 272 entries do not fit
//     next to the operands. A list is compacted (sorted, cut to its KK best) by merging 16-entry
//     chunks in registers, which happens rarely once the query's threshold has settled.
//
// Warps: 0 TMA producer, 1 MMA issuer (and TMEM owner), 2..5 epilogue (warp w reads TMEM lanes
// 32 * (w % 4) .. + 31; thread = query). Every mbarrier wait is bounded (a kernel argument); on
// timeout the CTA raises the launch's error word, drains its copies in flight (bounded), frees
// TMEM and exits, and the finalize sends every query to the exact rescan.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "qv_state.h"
#include "tc_common.cuh"

namespace qv {
namespace tcw {

using namespace qv::tc;

constexpr int kEpiWarps = 4;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr int kAcc = 2;           // accumulator slots of kN columns
constexpr int kLS = kM;           // list stride: entry i of query lane l at i * kLS + l
constexpr int kAppend = 16;       // entries appended between compactions (two 64-column halves)
constexpr int kMaxAtoms = 12;     // kpad <= 768
constexpr int kMaxStages = 12;
constexpr int kTmemAtoms = 8;     // query-tile K atoms held in TMEM (columns 256..511)
constexpr int kTmemCols = 512;
constexpr int kMaxKK = 256;       // longest best list (k up to 204)

struct Args {
  int nq, n_qtiles, n_chunks, total_units, atoms, stages, kk;
  int stage_atoms;          // K atoms of a row tile per ring stage (the tile's last may hold fewer)
  int a_tmem_atoms;         // leading K atoms of the query tile held in TMEM (the rest in smem)
  int kpad;
  const __half* q16;        // the queries' fp16 rows (kpad columns, zero rows past nq)
  int64_t nrows, chunk_rows;
  const float* qscale_inv;  // per query: 1 / (s_q * s_x)
  const float* qnorm2;      // per query ||q||^2 (L2)
  const float* xnorm2;      // per row ||x||^2 (L2)
  const uint64_t* bitmap;
  float* cand_d;
  uint32_t* cand_r;
  int* cand_n;
  unsigned* thr_bits;
  float* list_d;            // per CTA: (kk + kAppend) x kLS working lists
  uint32_t* list_r;
  int* err;
  long long wait_cycles;
  uint64_t drain_ns;
  int skip_fill;            // failure-detection test hook: CTA 0 skips this ring fill (-1: none)
  float ip_one;             // inner-product screen values are ip_one - <q,x> (1, or 0 for -<q,x>)
};

// Sorts 16 (distance, group) entries ascending in registers (bitonic network).
__device__ __forceinline__ void sort16(float (&d)[16], uint32_t (&r)[16]) {
#pragma unroll
  for (int size = 2; size <= 16; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        if ((lo & size) == 0)
          cex(d[lo], r[lo], d[hi], r[hi]);
        else
          cex(d[hi], r[hi], d[lo], r[lo]);
      }
    }
  }
}

// Keeps the best kk entries of a query's list (a sorted prefix of kk, then up to kAppend
// appended entries), sorted, and tightens the threshold to the kk-th. The appended entries are
// sorted in registers (carry), then merged into the prefix 16 entries at a time: the chunk and
// the carry (both sorted) form a 32-entry bitonic sequence; after a bitonic merge the lower 16
// are the chunk's new contents and the upper 16 the carry into the next chunk. The last carry
// (entries beyond kk) is dropped. The warp's lanes run the same fixed sequence (no divergence).
__device__ __noinline__ void compact_wide(float* d, uint32_t* r, int kk, int& cnt, float& thr) {
  const float kInf = __int_as_float(0x7f800000);
  float cd[16];
  uint32_t cr[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const bool in = kk + i < cnt;
    cd[i] = in ? d[(kk + i) * kLS] : kInf;
    cr[i] = in ? r[(kk + i) * kLS] : 0xffffffffu;
  }
  sort16(cd, cr);
  float last = kInf;
  for (int c = 0; c < kk; c += 16) {
    float xd[32];
    uint32_t xr[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      xd[i] = d[(c + i) * kLS];
      xr[i] = r[(c + i) * kLS];
      xd[31 - i] = cd[i];
      xr[31 - i] = cr[i];
    }
#pragma unroll
    for (int stride = 16; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        cex(xd[lo], xr[lo], xd[hi], xr[hi]);
      }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      d[(c + i) * kLS] = xd[i];
      r[(c + i) * kLS] = xr[i];
      cd[i] = xd[16 + i];
      cr[i] = xr[16 + i];
    }
    last = xd[15];
  }
  cnt = kk;
  thr = fminf(thr, last);
}

// One ring stage's MMAs: kAtomsN K atoms x 4 K steps, fully unrolled, with the descriptors
// advanced by constant offsets (a descriptor's start-address field is the byte address >> 4 in
// its low 14 bits, which a shared-memory address below 256 KB never carries out of). kTs: A from
// TMEM (a = its first column) or from shared memory (a = its byte address). first: the stage
// starts the tile's accumulation.
template <bool kPair, bool kTs, int kAtomsN, int kBAtomBytes>
__device__ __forceinline__ void issue_stage(uint32_t d_tmem, uint32_t a, uint32_t b_addr,
                                            bool first) {
  const uint64_t bd = smem_desc(b_addr);
  const uint64_t ad = kTs ? 0 : smem_desc(a);
#pragma unroll
  for (int i = 0; i < kAtomsN; ++i) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint32_t acc = (first && i == 0 && ks == 0) ? 0u : 1u;
      const uint64_t b = bd + static_cast<uint64_t>((i * kBAtomBytes + ks * 32) >> 4);
      if (kTs) {
        const uint32_t at = a + static_cast<uint32_t>(i * 32 + ks * 8);
        if (kPair)
          umma_f16_ts_pair(d_tmem, at, b, acc);
        else
          umma_f16_ts(d_tmem, at, b, acc);
      } else {
        const uint64_t ai = ad + static_cast<uint64_t>((i * kAtomBytes + ks * 32) >> 4);
        if (kPair)
          umma_f16_pair(d_tmem, ai, b, acc);
        else
          umma_f16(d_tmem, ai, b, acc);
      }
    }
  }
}

// kPair: the kernel runs as clusters of two CTAs (tcgen05 cta_group::2). A pair works on one
// unit at a time: a 256-query group (128 queries per CTA, each CTA's own A and its own best
// lists) against the unit's rows, each CTA loading 64 of every 128-row tile's rows; the even CTA
// (the leader) issues MMAs of M = 256, N = 128, so every row byte a CTA loads into shared memory
// feeds both CTAs' tensor cores. That halves the shared-memory traffic per MMA (the screen's
// limit with one CTA: ~128 B/clk of the SM's 128 B/clk for B's copies in and its reads out).
// Barriers both CTAs' producers, epilogues and copies report to (full, a_full, a_tfull,
// acc_empty, drain) live in the leader; the leader's commits arrive on both CTAs' copies of the
// others (empty, acc_full, a_empty) by multicast.
template <bool kL2, bool kPair>
__global__ void __launch_bounds__(kThreads, 1)
    flat_screen_tc_wide_kernel(const __grid_constant__ CUtensorMap tmap_q,
                               const __grid_constant__ CUtensorMap tmap_x, const Args a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int atoms = a.atoms, stages = a.stages, kk = a.kk, ta = a.a_tmem_atoms;
  const int sa = a.stage_atoms;
  // A row-tile K atom in shared memory: 128 rows (16 KB), or this CTA's 64 rows in a pair.
  constexpr int kBAtomBytes = kPair ? kAtomBytes / 2 : kAtomBytes;
  constexpr int kBRows = kPair ? kN / 2 : kN;
  unsigned char* smem_a = base;  // atoms - ta atoms x 16 KB (the query tile past TMEM's part)
  unsigned char* smem_b = smem_a + (atoms - ta) * kAtomBytes;  // stages x sa x kBAtomBytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_b + stages * sa * kBAtomBytes);
  // bars: full[stages], empty[stages], acc_full[kAcc], acc_empty[kAcc], a_full (smem part of
  // the query tile landed), a_empty (the unit's MMAs are done with the query tile), a_tfull
  // (the epilogue warps stored the TMEM part), drain (on abort, a final commit there tells
  // when the MMAs in flight have finished).
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ int s_consumed;  // B fills the MMA issuer has waited for (abort drain)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int FULL = 0, EMPTY = stages, ACC_FULL = 2 * stages, ACC_EMPTY = 2 * stages + kAcc,
            A_FULL = 2 * stages + 2 * kAcc, A_EMPTY = A_FULL + 1, A_TFULL = A_FULL + 2,
            DRAIN = A_FULL + 3;
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const uint32_t rank = kPair ? cluster_ctarank() : 0;
  const bool leader = rank == 0;
  // The leader's copy of barrier i, as a shared::cluster address (pair) or this CTA's (single).
  auto lbar = [&](int i) { return kPair ? mapa_shared(bar(i), 0) : bar(i); };
  auto wait = [&](uint32_t b, uint32_t parity, volatile int* abort_flag) {
    return kPair ? mbar_wait_cluster(b, parity, abort_flag, a.err, a.wait_cycles)
                 : mbar_wait(b, parity, abort_flag, a.err, a.wait_cycles);
  };
  auto arrive_leader = [&](int i) {
    if (kPair) {
      mbar_arrive_cluster(lbar(i));
    } else {
      mbar_arrive(bar(i));
    }
  };
  auto commit_both = [&](int i) {  // the MMAs issued so far have completed
    if (kPair) {
      umma_commit_pair_mc(bar(i), 0x3);
    } else {
      umma_commit(bar(i));
    }
  };

  if (threadIdx.x == 0) {
    s_abort = 0;
    s_consumed = 0;
    for (int s = 0; s < stages; ++s) {
      mbar_init(bar(FULL + s), 1);   // the (leader's) producer's expect_tx
      mbar_init(bar(EMPTY + s), 1);  // the MMA commit
    }
    for (int b = 0; b < kAcc; ++b) {
      mbar_init(bar(ACC_FULL + b), 1);
      mbar_init(bar(ACC_EMPTY + b), (kPair ? 2 : 1) * kEpiWarps);
    }
    mbar_init(bar(A_FULL), 1);
    mbar_init(bar(A_EMPTY), 1);
    mbar_init(bar(A_TFULL), (kPair ? 2 : 1) * kEpiWarps);
    mbar_init(bar(DRAIN), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if (kPair) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&s_tmem)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&s_tmem)),
                   "r"(kTmemCols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  if (kPair) cluster_sync();  // both CTAs' barriers are initialized before either uses them
  tc_fence_after();
  const uint32_t tmem_base = s_tmem;
  volatile int* abort_flag = &s_abort;

  // Units: (query group, row chunk), chunk-major so that CTAs running together share row chunks
  // in L2. A group is one 128-query tile, or two (one per CTA) in a pair.
  const int worker = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int workers = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int n_groups = kPair ? (a.n_qtiles + 1) / 2 : a.n_qtiles;
  auto unit_rows = [&](int u, int& qtile, int& chunk, int64_t& r0, int64_t& r1) {
    chunk = u / n_groups;
    const int group = u - chunk * n_groups;
    qtile = kPair ? 2 * group + static_cast<int>(rank) : group;
    r0 = static_cast<int64_t>(chunk) * a.chunk_rows;
    r1 = min(a.nrows, r0 + a.chunk_rows);
  };

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs of a pair) ----------------
    if (lane == 0) {
      int stage = 0, issued = 0;
      uint32_t phase = 0, a_phase = 0;
      bool first = true, ok = true;
      for (int u = worker; u < a.total_units && ok && !*abort_flag; u += workers) {
        int qtile, chunk;
        int64_t r0, r1;
        unit_rows(u, qtile, chunk, r0, r1);
        const int ntiles = static_cast<int>((r1 - r0 + kN - 1) / kN);
        if (!first) {
          if (!wait(bar(A_EMPTY), a_phase, abort_flag)) break;
          a_phase ^= 1;
        }
        first = false;
        // The query tile's atoms past the TMEM part (none when kpad <= 512: the arrival alone
        // completes the phase). In a pair, both CTAs' copies count on the leader's barrier.
        if (leader)
          mbar_expect_tx(bar(A_FULL),
                         static_cast<uint32_t>((kPair ? 2 : 1) * (atoms - ta) * kAtomBytes));
        for (int at = ta; at < atoms; ++at) {
          const uint32_t dst = smem_u32(smem_a + (at - ta) * kAtomBytes);
          if (kPair)
            tma_load_2d_pair(dst, &tmap_q, at * kAtomK, qtile * kM, lbar(A_FULL));
          else
            tma_load_2d(dst, &tmap_q, at * kAtomK, qtile * kM, bar(A_FULL));
        }
        for (int t = 0; t < ntiles && ok; ++t) {
          const int y = static_cast<int>(r0 + static_cast<int64_t>(t) * kN) +
                        static_cast<int>(rank) * kBRows;
          for (int at0 = 0; at0 < atoms; at0 += sa) {
            const int n_at = min(sa, atoms - at0);
            ok = wait(bar(EMPTY + stage), phase ^ 1, abort_flag);
            if (!ok) break;
            if (blockIdx.x != 0 || issued != a.skip_fill) {
              if (leader)
                mbar_expect_tx(bar(FULL + stage),
                               static_cast<uint32_t>((kPair ? 2 : 1) * n_at * kBAtomBytes));
              for (int i = 0; i < n_at; ++i) {
                const uint32_t dst = smem_u32(smem_b + (stage * sa + i) * kBAtomBytes);
                if (kPair)
                  tma_load_2d_pair(dst, &tmap_x, (at0 + i) * kAtomK, y, lbar(FULL + stage));
                else
                  tma_load_2d(dst, &tmap_x, (at0 + i) * kAtomK, y, bar(FULL + stage));
              }
            }
            ++issued;  // ring fills, the skipped one (test hook) included
            if (++stage == stages) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      if (*abort_flag) {
        const uint64_t t0 = gtimer();
        if (kPair) {
          // A pair's copies complete on the leader's barriers, which the peer cannot poll: wait
          // out the drain bound, far longer than any copy in flight takes.
          while (gtimer() - t0 < a.drain_ns) {
          }
        } else {
          // Wait (bounded) for every B fill the MMA issuer did not consume: each fill's barrier
          // phase completes when its bytes have landed.
          for (int f = *reinterpret_cast<volatile int*>(&s_consumed); f < issued; ++f) {
            if (blockIdx.x == 0 && f == a.skip_fill) continue;
            const int s = f % stages;
            const uint32_t par = (f / stages) & 1;
            while (!mbar_test(bar(FULL + s), par) && gtimer() - t0 < a.drain_ns) {
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (the leader of a pair) ----------------
    if (lane == 0 && leader) {
      int stage = 0, g = 0;  // g: row tiles issued by this CTA so far (slot g & 1)
      uint32_t phase = 0, a_phase = 0;
      bool ok = true;
      for (int u = worker; u < a.total_units && ok && !*abort_flag; u += workers) {
        int qtile, chunk;
        int64_t r0, r1;
        unit_rows(u, qtile, chunk, r0, r1);
        const int ntiles = static_cast<int>((r1 - r0 + kN - 1) / kN);
        if (!wait(bar(A_FULL), a_phase, abort_flag)) break;
        if (!wait(bar(A_TFULL), a_phase, abort_flag)) break;
        a_phase ^= 1;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem_a);
        const uint32_t a_tmem = tmem_base + static_cast<uint32_t>(kAcc * kN);
        for (int t = 0; t < ntiles && ok; ++t, ++g) {
          const int slot = g & 1;
          // The slot's previous tile (g - 2) must have been read out by the epilogue(s).
          ok = wait(bar(ACC_EMPTY + slot), ((g >> 1) & 1) ^ 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(slot * kN);
          for (int at0 = 0; at0 < atoms; at0 += sa) {
            const int n_at = min(sa, atoms - at0);
            ok = wait(bar(FULL + stage), phase, abort_flag);
            if (!ok) break;
            *reinterpret_cast<volatile int*>(&s_consumed) += 1;
            // No tcgen05 fence here: the stage's bytes come from the TMA (async proxy) and its
            // barrier's completion orders them before the MMAs that read them; only the TMEM
            // hand-offs between threads (accumulator slot, query tile) need the fence.
            const uint32_t b_stage = smem_u32(smem_b + stage * sa * kBAtomBytes);
            if (n_at == 4 && (at0 + 4 <= ta || at0 >= ta)) {
              // The common case: four atoms all from TMEM or all from shared memory.
              if (at0 < ta)
                issue_stage<kPair, true, 4, kBAtomBytes>(
                    d_tmem, a_tmem + static_cast<uint32_t>(at0 * 32), b_stage, at0 == 0);
              else
                issue_stage<kPair, false, 4, kBAtomBytes>(
                    d_tmem, a_addr + static_cast<uint32_t>((at0 - ta) * kAtomBytes), b_stage,
                    at0 == 0);
            } else {
              for (int i = 0; i < n_at; ++i) {
                const int at = at0 + i;
                const uint32_t b_addr = b_stage + static_cast<uint32_t>(i * kBAtomBytes);
                if (at < ta)  // A from TMEM: 64 fp16 per atom = 32 columns, 8 per K step
                  issue_stage<kPair, true, 1, kBAtomBytes>(
                      d_tmem, a_tmem + static_cast<uint32_t>(at * 32), b_addr, at == 0);
                else
                  issue_stage<kPair, false, 1, kBAtomBytes>(
                      d_tmem, a_addr + static_cast<uint32_t>((at - ta) * kAtomBytes), b_addr,
                      at == 0);
              }
            }
            commit_both(EMPTY + stage);  // the stage is free once these MMAs have read it
            if (++stage == stages) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          commit_both(ACC_FULL + slot);
        }
        if (!ok) break;
        commit_both(A_EMPTY);  // the query tile may be replaced once every MMA has run
      }
      if (*abort_flag) {
        // Wait (bounded) for the MMAs in flight before the accumulators are freed.
        if (kPair)
          umma_commit_pair_mc(bar(DRAIN), 0x1);
        else
          umma_commit(bar(DRAIN));
        const uint64_t t0 = gtimer();
        while (!mbar_test(bar(DRAIN), 0) && gtimer() - t0 < a.drain_ns) {
        }
      }
    }
  } else {
    // ---------------- epilogue: thread = query (both CTAs of a pair) ----------------
    const int quarter = warp & 3;  // TMEM lanes this warp may read
    const int qi = quarter * 32 + lane;
    float* ld = a.list_d + static_cast<size_t>(blockIdx.x) * (kk + kAppend) * kLS + qi;
    uint32_t* lr = a.list_r + static_cast<size_t>(blockIdx.x) * (kk + kAppend) * kLS + qi;
    const int cap = kk + kAppend;
    const float kInfF = __int_as_float(0x7f800000);
    int g = 0;
    uint32_t a_phase = 0;
    bool ok = true, first = true;
    for (int u = worker; u < a.total_units && ok; u += workers) {
      int qtile, chunk;
      int64_t r0, r1;
      unit_rows(u, qtile, chunk, r0, r1);
      const int ntiles = static_cast<int>((r1 - r0 + kN - 1) / kN);
      const int q = qtile * kM + qi;
      // The query tile's first ta atoms into this warp's 32 TMEM lanes (columns 256 + 32 * atom),
      // once the previous unit's MMAs have finished reading them.
      if (!first) {
        ok = wait(bar(A_EMPTY), a_phase, abort_flag);
        if (!ok) break;
        a_phase ^= 1;
        tc_fence_after();
      }
      first = false;
      {
        const uint4* row = reinterpret_cast<const uint4*>(
            a.q16 + static_cast<size_t>(qtile * kM + qi) * a.kpad);
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(kAcc * kN);
        for (int at = 0; at < ta; ++at) {
          uint32_t w[32];
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            const int h = at * kAtomK + v * 8;  // first fp16 element of this 16-byte piece
            const uint4 x = h < a.kpad ? __ldg(row + h / 8) : make_uint4(0, 0, 0, 0);
            w[4 * v] = x.x;
            w[4 * v + 1] = x.y;
            w[4 * v + 2] = x.z;
            w[4 * v + 3] = x.w;
          }
          tmem_st32(tbase + static_cast<uint32_t>(at * 32), w);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_leader(A_TFULL);
      }
      const bool active = q < a.nq;
      const unsigned* qthr = a.thr_bits + (active ? q : 0);
      float thr = active ? dev::from_ordered_bits(*qthr) : -kInfF;
      const float inv = active ? a.qscale_inv[q] : 0.0f;
      const float qn = (active && kL2) ? a.qnorm2[q] : 0.0f;
      for (int i = 0; i < kk; ++i) {
        ld[i * kLS] = kInfF;
        lr[i * kLS] = 0xffffffffu;
      }
      int cnt = kk, seen = 0;
      // best[j]: best score of the 8-row group j of a 64-column half (max inner product for
      // cosine/IP, min distance for L2); rows past the chunk or rejected by the filter count as
      // the worst score.
      auto tree = [&](uint32_t (&r)[64], int64_t cb, float (&best)[8], float& top) {
        float (&v)[64] = *reinterpret_cast<float(*)[64]>(r);
        const bool partial = a.bitmap != nullptr || r1 - cb < 64;
        uint64_t admitted = ~0ull;
        if (partial) {
          const int valid = static_cast<int>(r1 - cb < 64 ? r1 - cb : 64);
          admitted = (valid >= 64 ? ~0ull : (valid > 0 ? (1ull << valid) - 1 : 0ull)) &
                     (a.bitmap != nullptr && valid > 0 ? a.bitmap[static_cast<uint64_t>(cb) >> 6]
                                                       : ~0ull);
        }
        if (kL2) {
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const bool in = (admitted >> j) & 1ull;
            const float xn = in ? a.xnorm2[cb + j] : 0.0f;
            v[j] = in ? fmaf(-2.0f * inv, v[j], qn + xn) : kInfF;
          }
          group_best8<false>(v, best, top);
        } else {
          if (admitted != ~0ull) {
#pragma unroll
            for (int j = 0; j < 64; ++j)
              if (!((admitted >> j) & 1ull)) v[j] = -kInfF;
          }
          group_best8<true>(v, best, top);
        }
      };
      auto screen = [&](const float (&best)[8], float top, int64_t cb) {
        const bool may = active && screen_value<kL2>(top, inv, a.ip_one) <= thr;
        if (!__any_sync(0xffffffffu, may)) return;
        uint32_t gm = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          gm |= (may && screen_value<kL2>(best[j], inv, a.ip_one) <= thr) ? (1u << j) : 0u;
        if (__any_sync(0xffffffffu, cnt + __popc(gm) > cap)) {
          compact_wide(ld, lr, kk, cnt, thr);
          if (active) atomicMin(a.thr_bits + q, dev::ordered_bits(thr));
          uint32_t keep = 0;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            keep |= (screen_value<kL2>(best[j], inv, a.ip_one) <= thr) ? (1u << j) : 0u;
          gm &= keep;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if ((gm >> j) & 1u) {
            const int pos = cnt + __popc(gm & ((1u << j) - 1u));
            ld[pos * kLS] = screen_value<kL2>(best[j], inv, a.ip_one);
            lr[pos * kLS] = static_cast<uint32_t>(cb / kTcGroupRows + j);
          }
        }
        const int np = __popc(gm);
        cnt += np;
        seen += np;
      };
      uint32_t ra[64], rb[64];
      unsigned fresh = ~0u;
      for (int t = 0; t < ntiles; ++t, ++g) {
        const int slot = g & 1;
        const int64_t row0 = r0 + static_cast<int64_t>(t) * kN;
        if ((t & 7) == 0 && active) fresh = *reinterpret_cast<const volatile unsigned*>(qthr);
        ok = wait(bar(ACC_FULL + slot), (g >> 1) & 1, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t taddr =
            tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(slot * kN);
        tmem_ld64_issue(taddr, ra);
        tmem_ld64_issue(taddr + 64, rb);
        tmem_wait_ld(ra);
        tmem_hold(rb);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) arrive_leader(ACC_EMPTY + slot);
        float best_a[8], best_b[8], top_a, top_b;
        tree(ra, row0, best_a, top_a);
        tree(rb, row0 + 64, best_b, top_b);
        screen(best_a, top_a, row0);
        screen(best_b, top_b, row0 + 64);
        if ((t & 7) == 7) thr = fminf(thr, dev::from_ordered_bits(fresh));
      }
      if (!ok) break;
      compact_wide(ld, lr, kk, cnt, thr);
      cnt = min(seen, kk);
      if (active) {
        const size_t slot = static_cast<size_t>(q) * a.n_chunks + chunk;
        for (int i = 0; i < cnt; ++i) {
          a.cand_d[slot * kk + i] = ld[i * kLS];
          a.cand_r[slot * kk + i] = lr[i * kLS];
        }
        a.cand_n[slot] = cnt;
        if (cnt == kk) atomicMin(a.thr_bits + q, dev::ordered_bits(ld[(kk - 1) * kLS]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // In a pair, neither CTA frees its tensor memory or leaves while the other may still reach
  // its barriers or the leader's MMAs its memory.
  if (kPair) cluster_sync();
  tc_fence_after();
  if (warp == 1) {
    if (kPair) {
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(kTmemCols));
    } else {
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(kTmemCols));
    }
  }
}

}  // namespace tcw

// ---- host side ------------------------------------------------------------------------------------

// Best-list length of the wide screen: k plus a margin of max(8, k / 4) groups, in whole 16-entry
// chunks. The certificate needs the list's last value to clear the k-th exact distance by the
// screen's error bound; for large k over dense data (768-dim inner product, k = 100) the
// distances near rank k are packed so closely that a margin of 8 left about one query in eight
// uncertified, while k / 4 clears it by several error bounds.
int flat_tc_wide_kk(size_t k) {
  return static_cast<int>(ceil_div(k + std::max<size_t>(8, (k + 3) / 4), 16) * 16);
}

bool flat_tc_wide_fits(const FlatState& s, size_t k) {
  const size_t kpad = std::max<size_t>(64, ceil_div(s.dim, 16) * 16);
  return ceil_div(kpad, tc::kAtomK) <= static_cast<size_t>(tcw::kMaxAtoms) &&
         flat_tc_wide_kk(k) <= tcw::kMaxKK;
}

size_t flat_tc_wide_list_bytes(const FlatState& s, int kk) {
  return static_cast<size_t>(sm_count(s.device)) * (kk + tcw::kAppend) * tcw::kLS * 8;
}

void flat_screen_tc_wide(const FlatState& s, const float* qp, int dpad, size_t nq,
                         const uint64_t* d_bitmap, int n_chunks, int64_t chunk_rows, int kk,
                         float* cand_d, uint32_t* cand_r, int* cand_n, unsigned* thr_bits,
                         float* eps, int* err, const CUtensorMap& mq, const __half* q16,
                         const float* qinv, const float* qn2, void* lists, cudaStream_t st) {
  QV_REQUIRE(kk % 16 == 0 && kk <= tcw::kMaxKK,
             "wide tensor-core screen: unsupported best-list length");
  const int kpad = static_cast<int>(s.kpad);
  const int atoms = static_cast<int>(ceil_div(static_cast<size_t>(kpad), tc::kAtomK));
  QV_REQUIRE(atoms <= tcw::kMaxAtoms, "wide tensor-core screen: rows wider than 768");
  // Single CTAs unless QV_TC_WIDE_PAIR=1 selects CTA pairs (tcgen05 cta_group::2). On the 768-dim
  // workload (16,384 queries x 5M rows, power-capped clocks) both ran in 165-200 M SM cycles
  // against a 104 M-cycle MMA floor; pairs halve the L2-to-SM traffic but did not run faster.
  const char* pe = std::getenv("QV_TC_WIDE_PAIR");
  const bool pair = pe != nullptr && pe[0] == '1';
  const int nsm = sm_count(s.device);
  // A pair's CTAs each load 64 rows of every 128-row tile.
  const CUtensorMap mx = tc::make_map(s.x16.get(), s.n, kpad, pair ? tc::kN / 2 : tc::kN);
  tcw::Args a{};
  a.nq = static_cast<int>(nq);
  a.n_qtiles = static_cast<int>(ceil_div(nq, tc::kM));
  a.n_chunks = n_chunks;
  a.total_units = (pair ? (a.n_qtiles + 1) / 2 : a.n_qtiles) * n_chunks;
  a.atoms = atoms;
  a.kk = kk;
  a.nrows = static_cast<int64_t>(s.n);
  a.chunk_rows = chunk_rows;
  a.qscale_inv = qinv;
  a.qnorm2 = qn2;
  a.xnorm2 = s.xnorm2.get<float>();
  a.bitmap = d_bitmap;
  a.cand_d = cand_d;
  a.cand_r = cand_r;
  a.cand_n = cand_n;
  a.thr_bits = thr_bits;
  a.list_d = static_cast<float*>(lists);
  const int grid = pair ? 2 * std::min(a.total_units, nsm / 2) : std::min(a.total_units, nsm);
  a.list_r = reinterpret_cast<uint32_t*>(static_cast<float*>(lists) +
                                         static_cast<size_t>(grid) * (kk + tcw::kAppend) * tcw::kLS);
  a.err = err;
  a.wait_cycles = tc::wait_limit_cycles();
  a.drain_ns = tc::drain_limit_ns();
  a.skip_fill = tc::test_skip_fill();
  a.ip_one = s.neg_ip ? 0.0f : 1.0f;
  a.a_tmem_atoms = std::min(atoms, tcw::kTmemAtoms);
  a.kpad = kpad;
  a.q16 = q16;
  // Shared memory: the query tile's atoms past TMEM's part, a ring of row-tile K atoms (16 KB, or
  // 8 KB for a pair's 64-row halves), barriers; never less than half the SM's shared memory, so
  // that one CTA (and its 512 TMEM columns) runs per SM.
  constexpr size_t kSmemMax = 227 * 1024 - 1024;  // per block, less the kernel's static part
  const size_t b_atom = pair ? tc::kAtomBytes / 2 : tc::kAtomBytes;
  const size_t fixed = 1024 + static_cast<size_t>(atoms - a.a_tmem_atoms) * tc::kAtomBytes + 256;
  const size_t room = (kSmemMax - fixed) / b_atom;  // row-tile K atoms the ring can hold
  // Four atoms per stage (sixteen MMAs per barrier wait in the issuing thread) while that still
  // leaves two stages: on the 768-dim workload (single CTAs) one-, two-, three- and four-atom
  // stages took 311, 238, 202 and 202 M SM cycles per 16,384 x 5M batch.
  // QV_TC_WIDE_STAGE_ATOMS (1..4) overrides.
  int sa = room >= 8 ? 4 : (room >= 4 ? 2 : 1);
  if (const char* e = std::getenv("QV_TC_WIDE_STAGE_ATOMS"); e != nullptr && *e != '\0')
    sa = std::max(1, std::min(4, std::atoi(e)));
  sa = std::min(sa, atoms);
  const int stages = static_cast<int>(std::min<size_t>(tcw::kMaxStages, room / sa));
  QV_REQUIRE(stages >= 2, "wide tensor-core screen: no room for two row stages");
  a.stages = stages;
  a.stage_atoms = sa;
  const size_t smem =
      std::max<size_t>(fixed + static_cast<size_t>(stages) * sa * b_atom, 120 * 1024);
  KernelTimer timer(st, "flat_screen_tc_wide_kernel",
                    2.0 * nq * static_cast<double>(s.n) * s.dim, false);
  const bool l2 = s.metric == QV_METRIC_L2;
  if (pair) {
    auto kernel = l2 ? tcw::flat_screen_tc_wide_kernel<true, true>
                     : tcw::flat_screen_tc_wide_kernel<false, true>;
    QV_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(tcw::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QV_CUDA(cudaLaunchKernelEx(&cfg, kernel, mq, mx, a));
  } else {
    auto kernel = l2 ? tcw::flat_screen_tc_wide_kernel<true, false>
                     : tcw::flat_screen_tc_wide_kernel<false, false>;
    QV_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kernel<<<grid, tcw::kThreads, smem, st>>>(mq, mx, a);
  }
  timer.stop();
  check_launch("flat_screen_tc_wide_kernel");
  (void)eps;
}

}  // namespace qv
