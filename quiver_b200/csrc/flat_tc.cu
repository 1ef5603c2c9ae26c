// Tensor-core (tcgen05) screen for exact Flat search on sm_100a.
//
// The screen computes every query-row inner product with one fp16 MMA pass: queries and rows are
// converted to float16 (times a power-of-two scale, which is exact, only when their magnitudes
// need it), multiplied on the 5th-generation tensor cores with float32 accumulation in TMEM, and
// each query keeps its KK best screen candidates. The exact re-rank and the certificate in
// flat.cu then make the final result identical to the reference's: the float16 rounding errors
// enter a rigorous per-query bound (measured ||q - q16|| and max ||x - x16||, plus accumulation
// and reference rounding), and any query whose candidate set cannot be proven complete is
// rescanned exactly.
//
// Kernel structure (one CTA per SM, persistent over work units = (query group of 2 x 128, row
// chunk), chunk-major so that the CTAs working on a chunk share its rows in L2):
//   warp 0      TMA producer: the unit's two query tiles (A, resident) and a ring of 128-row tiles
//               of the database (B; 3 stages with best lists of 24, else 2), 128-byte swizzled, no
//               multicast.
//   warps 1, 10 MMA issuers (even / odd row tiles): tcgen05.mma kind::f16 (M=128, N=128, K=16
//               steps, unrolled per K-step count) of each row tile against both query tiles into
//               one of two TMEM accumulator slots (2 x 128 columns each); one mbarrier wait per
//               tile, which covers both the tile's bytes and its slot being free.
//   warps 2..9  epilogue: warp (tile, lane quarter); thread i owns query i of its tile (= TMEM
//               lane), loads the tile's 128 inner products, frees the slot, reduces each 8-row group
//               to its best score with three-input max/min trees, and appends the groups that beat
//               its running threshold to a candidate list in shared memory (compacted in registers
//               by fixed sorting networks when one fills).
// Every mbarrier wait is bounded (2 s of GPU time); on timeout the CTA raises an error flag,
// drains its outstanding copies (again bounded), frees TMEM and exits.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "qv_state.h"
#include "tc_common.cuh"

namespace qv {
namespace tc {

constexpr int kTiles = 2;        // query tiles per CTA: every row tile feeds one MMA per query tile
constexpr int kEpiWarps = 4 * kTiles;  // one warp per (query tile, TMEM lane quarter)
// Warps: 0 TMA producer, 1 MMA issuer of even row tiles, 2 .. 1 + kEpiWarps epilogue, and
// kIssuer2 MMA issuer of odd row tiles. Each mbarrier wait in an issuing thread leaves the tensor
// pipe idle for ~200 cycles; with two issuers one waits while the other's MMAs run.
constexpr int kIssuer2 = 2 + kEpiWarps;
constexpr int kThreads = 32 * (kIssuer2 + 1);
constexpr int kAcc = 2;          // TMEM accumulator slots of kTiles x kN columns (all 512 columns)
constexpr int kLS = kTiles * kM; // candidate-list stride: entry i of list l lives at i * kLS + l
constexpr int kMaxKK = 32;       // largest best-list length (candidates per query per unit)
constexpr int kMergeTries = 256; // attempts to take a query's running-list lock at a unit's end
// Row-tile ring depth and list entries appended between compactions, by best-list length. A row
// tile's stage is only refilled after its MMAs finish, so the next tile's copy has one tile time
// (~900 cycles) to land with two stages, which L2 latency exceeds; three stages fit in shared
// memory next to best lists of 24 when 8 (not 16) entries are appended between compactions.
// In CTA pairs (kPair) a CTA holds only half of each row tile (64 rows, 8 KB per K atom), which
// leaves room for a deeper ring and longer append runs (fewer list compactions).
template <int kKK, bool kPair = false, int kAtoms = 2>
struct Ring {
  static constexpr int kStages = kPair ? (kAtoms == 1 ? 8 : (kKK <= 24 ? 5 : 4))
                                       : (kKK <= 24 ? 3 : 2);
  static constexpr int kAppend = kPair ? 16 : (kKK <= 24 ? 8 : 16);
};
struct Args {
  int nq, n_qgroups, n_chunks, total_units, ksteps;  // a query group = kTiles tiles of kM
  int64_t nrows, chunk_rows;
  bool l2;
  const float* qscale_inv;  // per query: 1 / (s_q * s_x)
  const float* qnorm2;      // per query ||q||^2 (L2)
  const float* xnorm2;      // per row ||x||^2 (L2)
  const uint64_t* bitmap;
  float* cand_d;
  uint32_t* cand_r;
  int* cand_n;
  unsigned* thr_bits;
  float* gbest;     // nq x kMaxKK: the KK best distances output by the query's finished
                    // units, sorted, padded with +inf
  int* glock;       // nq: try-lock guarding gbest[q]
  int* err;
  bool qmajor;      // unit order: query-tile-major (true) or row-chunk-major (false)
  long long wait_cycles;  // bound of every mbarrier wait (SM clock cycles)
  uint64_t drain_ns;      // bound of the abort path's waits for work in flight (global timer)
  int skip_fill;          // failure-detection test hook: CTA 0 skips this ring fill (-1: none)
  float ip_one;           // inner-product screen values are ip_one - <q,x> (1, or 0 for -<q,x>)
  // Threshold seeding launch: units only publish their lists' kKK-th values as the queries'
  // thresholds (no candidate lists, no running best-list merge).
  bool seed_only;
};

__device__ __forceinline__ void unit_coords(const Args& a, int u, int& qgroup, int& chunk) {
  if (a.qmajor) {
    qgroup = u / a.n_chunks;
    chunk = u - qgroup * a.n_chunks;
  } else {
    chunk = u / a.n_qgroups;
    qgroup = u - chunk * a.n_qgroups;
  }
}

// Keeps the best kKK of a query's list, sorted, and tightens the threshold to the kKK-th distance
// (+inf while fewer than kKK real entries were seen). The list is loaded into registers and
// merged there by fixed networks (no per-lane branches, so the warp never diverges): the appended
// entries (padded with (+inf, ~0)) are sorted by a kAppend-input bitonic network; with the prefix
// a (sorted, padded to 32) and the sorted appended entries b (padded to 32), c[i] = min(a[i],
// b[31 - i]) holds the 32 smallest of both as a bitonic sequence, which a 32-input bitonic merge
// sorts.
template <int kKK, int kA>
__device__ __noinline__ void compact_buffer(float* d, uint32_t* r, int& cnt, float& thr) {
  static_assert((kA & (kA - 1)) == 0 && kA <= 32 && kKK <= 32, "networks sized for 32 kept");
  const float kInf = __int_as_float(0x7f800000);
  float bd[kA];
  uint32_t br[kA];
#pragma unroll
  for (int i = 0; i < kA; ++i) {
    const bool in = kKK + i < cnt;
    bd[i] = in ? d[(kKK + i) * kLS] : kInf;
    br[i] = in ? r[(kKK + i) * kLS] : 0xffffffffu;
  }
#pragma unroll
  for (int size = 2; size <= kA; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < kA / 2; ++i) {
        const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        if ((lo & size) == 0)
          cex(bd[lo], br[lo], bd[hi], br[hi]);
        else
          cex(bd[hi], br[hi], bd[lo], br[lo]);
      }
    }
  }
  float cd[32];
  uint32_t cr[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    cd[i] = i < kKK ? d[i * kLS] : kInf;
    cr[i] = i < kKK ? r[i * kLS] : 0xffffffffu;
    if (31 - i < kA) {
      const bool tb = dev::key_less(bd[31 - i], br[31 - i], cd[i], cr[i]);
      cd[i] = tb ? bd[31 - i] : cd[i];
      cr[i] = tb ? br[31 - i] : cr[i];
    }
  }
#pragma unroll
  for (int stride = 16; stride > 0; stride >>= 1) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
      cex(cd[lo], cr[lo], cd[hi], cr[hi]);
    }
  }
#pragma unroll
  for (int i = 0; i < kKK; ++i) {
    d[i * kLS] = cd[i];
    r[i * kLS] = cr[i];
  }
  cnt = kKK;
  thr = fminf(thr, cd[kKK - 1]);
}

// One row tile's MMAs against every query tile of the group, kSteps K-steps of 16 each, fully
// unrolled: issued from a loop with a runtime trip count, each MMA took longer to issue than the
// 64 cycles a 128 x 128 x 16 MMA executes in, and even a guarded unrolled loop cost ~10 %.
// kPair: MMAs of M = 256 (cta_group::2, issued by the pair's leader), B's K atoms being this
// CTA's 64-row halves (8 KB apart instead of 16 KB).
template <int kAtoms, int kSteps, bool kPair>
__device__ __forceinline__ void issue_tile(uint32_t d_base, uint32_t a_addr, uint32_t b_addr) {
  constexpr int kBAtom = kPair ? kAtomBytes / 2 : kAtomBytes;
#pragma unroll
  for (int tq = 0; tq < kTiles; ++tq) {
#pragma unroll
    for (int ks = 0; ks < kSteps; ++ks) {
      const uint32_t off_a = static_cast<uint32_t>((ks >> 2) * kAtomBytes + (ks & 3) * 32);
      const uint32_t off_b = static_cast<uint32_t>((ks >> 2) * kBAtom + (ks & 3) * 32);
      const uint64_t da = smem_desc(a_addr + static_cast<uint32_t>(tq * kAtoms * kAtomBytes) + off_a);
      const uint64_t db = smem_desc(b_addr + off_b);
      if (kPair)
        umma_f16_pair(d_base + static_cast<uint32_t>(tq * kN), da, db, ks > 0 ? 1u : 0u);
      else
        umma_f16(d_base + static_cast<uint32_t>(tq * kN), da, db, ks > 0 ? 1u : 0u);
    }
  }
}

// kPair: the kernel runs as clusters of two CTAs (tcgen05 cta_group::2). A pair works on units of
// a 512-query group (two 128-query tiles per CTA, each CTA's own A, lists and accumulators)
// against a row chunk; each CTA loads 64 rows of every 128-row tile, and the even CTA (the
// leader) issues MMAs of M = 256 (both CTAs' query tile tq) x N = 128, so every row byte a CTA
// brings into shared memory feeds both tensor cores: per MMA an SM reads 6 KB of shared memory
// (its 4 KB of A, its 2 KB of B) instead of 8 KB, the copies in halve, and the ring covers twice
// the time for the same bytes. Barriers that both CTAs report to (full, a_full, drain) live in the
// leader; the leader's commits arrive on both CTAs' copies of empty, acc_full and a_empty.
template <int kAtoms, bool kL2, int kKK, bool kPair>
__global__ void __launch_bounds__(kThreads, 1)
    flat_screen_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                          const __grid_constant__ CUtensorMap tmap_x, const Args a) {
  constexpr int kStages = Ring<kKK, kPair, kAtoms>::kStages;
  constexpr int kAppend = Ring<kKK, kPair, kAtoms>::kAppend;
  constexpr int kCap = kKK + kAppend;  // candidate list entries per query
  constexpr int kBAtomBytes = kPair ? kAtomBytes / 2 : kAtomBytes;  // one row-tile K atom here
  constexpr int kBRows = kPair ? kN / 2 : kN;                       // rows of a tile loaded here
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the swizzle atoms.
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* smem_a = base;                                  // kTiles x kAtoms x 16 KB
  unsigned char* smem_b = smem_a + kTiles * kAtoms * kAtomBytes;  // kStages x kAtoms x kBAtomBytes
  float* buf_d = reinterpret_cast<float*>(smem_b + kStages * kAtoms * kBAtomBytes);  // kCap x kLS
  uint32_t* buf_r = reinterpret_cast<uint32_t*>(buf_d + kCap * kLS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(buf_r + kCap * kLS);
  // bars: full[kStages], empty[kStages], acc_full[kAcc], a_full, a_empty, drain[2] (one per
  // issuer: on abort, a final commit there tells when its MMAs in flight have finished).
  // Row tile t (counted over all of this CTA's units) uses stage t % kStages and accumulator slot
  // t % kAcc. full[t % kStages] also stands for "slot t % kAcc is free": it completes only when
  // the tile's bytes have landed AND every epilogue warp has read tile t - kAcc out of the slot
  // (the epilogue arrives on the stage of tile t + kAcc right after loading tile t). The MMA
  // issuers then wait on one mbarrier per tile: each wait in an issuing thread costs the tensor
  // pipe ~200 cycles of idle time, even on a phase that completed long before.
  static_assert(kStages >= kAcc, "an epilogue arrival must never reach a phase still in use");
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ int s_consumed[2];  // B fills each MMA issuer has waited for (abort drain)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int FULL = 0, EMPTY = kStages, ACC_FULL = 2 * kStages, A_FULL = 2 * kStages + kAcc,
            A_EMPTY = 2 * kStages + kAcc + 1, DRAIN = 2 * kStages + kAcc + 2;
  const uint32_t rank = kPair ? cluster_ctarank() : 0;
  const bool leader = rank == 0;
  // The leader's copy of barrier i (a shared::cluster address in a pair).
  auto lbar = [&](int i) { return kPair ? mapa_shared(bar(i), 0) : bar(i); };
  auto wait = [&](uint32_t b, uint32_t parity, volatile int* abort_flag) {
    return kPair ? mbar_wait_cluster(b, parity, abort_flag, a.err, a.wait_cycles)
                 : mbar_wait(b, parity, abort_flag, a.err, a.wait_cycles);
  };
  auto arrive_leader = [&](int i) {
    if (kPair)
      mbar_arrive_cluster(lbar(i));
    else
      mbar_arrive(bar(i));
  };
  auto commit_both = [&](int i) {  // the MMAs issued so far have completed
    if (kPair)
      umma_commit_pair_mc(bar(i), 0x3);
    else
      umma_commit(bar(i));
  };

  if (threadIdx.x == 0) {
    s_abort = 0;
    s_consumed[0] = s_consumed[1] = 0;
    for (int s = 0; s < kStages; ++s) {
      // The (leader's) producer's expect_tx + each epilogue warp (of both CTAs in a pair).
      mbar_init(bar(FULL + s), 1 + (kPair ? 2 : 1) * kEpiWarps);
      mbar_init(bar(EMPTY + s), 1);
    }
    for (int b = 0; b < kAcc; ++b) mbar_init(bar(ACC_FULL + b), 1);
    mbar_init(bar(A_FULL), 1);
    mbar_init(bar(A_EMPTY), 2);  // one commit per MMA issuer
    mbar_init(bar(DRAIN), 1);
    mbar_init(bar(DRAIN + 1), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    if (kPair) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&s_tmem)),
                   "r"(kAcc * kTiles * kN));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&s_tmem)),
                   "r"(kAcc * kTiles * kN));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  tc_fence_before();
  __syncthreads();
  if (kPair) cluster_sync();  // both CTAs' barriers are initialized before either uses them
  tc_fence_after();
  const uint32_t tmem_base = s_tmem;
  volatile int* abort_flag = &s_abort;
  // Work units (query group, row chunk): a group is kTiles query tiles, or 2 x kTiles in a pair
  // (CTA rank r holds tiles 2r .. 2r + 1 of the group). Pairs are numbered by blockIdx.x / 2.
  const int worker = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int workers = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  auto first_tile = [&](int qgroup) {  // this CTA's first query tile of the group
    return (kPair ? 2 * qgroup + static_cast<int>(rank) : qgroup) * kTiles;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, a_phase = 0;
      int issued = 0;
      bool first = true;
      for (int u = worker; u < a.total_units && !*abort_flag; u += workers) {
        int qgroup, chunk;
        unit_coords(a, u, qgroup, chunk);
        const int64_t r0 = static_cast<int64_t>(chunk) * a.chunk_rows;
        const int64_t r1 = min(a.nrows, r0 + a.chunk_rows);
        const int ntiles = static_cast<int>((r1 - r0 + kN - 1) / kN);
        if (!first) {
          if (!wait(bar(A_EMPTY), a_phase, abort_flag)) break;
          a_phase ^= 1;
        }
        first = false;
        // In a pair both CTAs' query tiles complete on the leader's barrier.
        if (leader) mbar_expect_tx(bar(A_FULL), (kPair ? 2 : 1) * kTiles * kAtoms * kAtomBytes);
        const int qt0 = first_tile(qgroup);
        for (int tq = 0; tq < kTiles; ++tq)
          for (int at = 0; at < kAtoms; ++at) {
            const uint32_t dst = smem_u32(smem_a + (tq * kAtoms + at) * kAtomBytes);
            if (kPair)
              tma_load_2d_pair(dst, &tmap_q, at * kAtomK, (qt0 + tq) * kM, lbar(A_FULL));
            else
              tma_load_2d(dst, &tmap_q, at * kAtomK, (qt0 + tq) * kM, bar(A_FULL));
          }
        for (int t = 0; t < ntiles; ++t) {
          if (!wait(bar(EMPTY + stage), phase ^ 1, abort_flag)) break;
          if (blockIdx.x != 0 || issued != a.skip_fill) {
            if (leader)
              mbar_expect_tx(bar(FULL + stage), (kPair ? 2 : 1) * kAtoms * kBAtomBytes);
            unsigned char* dst = smem_b + stage * kAtoms * kBAtomBytes;
            const int y = static_cast<int>(r0 + static_cast<int64_t>(t) * kN) +
                          static_cast<int>(rank) * kBRows;
            for (int at = 0; at < kAtoms; ++at) {
              if (kPair)
                tma_load_2d_pair(smem_u32(dst + at * kBAtomBytes), &tmap_x, at * kAtomK, y,
                                 lbar(FULL + stage));
              else
                tma_load_2d(smem_u32(dst + at * kBAtomBytes), &tmap_x, at * kAtomK, y,
                            bar(FULL + stage));
            }
          }
          ++issued;  // ring fills, the skipped one (test hook) included
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (*abort_flag && kPair) {
        // A pair's copies complete on the leader's barriers, which the peer cannot poll: wait
        // out the drain bound, far longer than any copy in flight takes.
        const uint64_t t0 = gtimer();
        while (gtimer() - t0 < a.drain_ns) {
        }
      } else if (*abort_flag) {
        // Drain: wait (bounded) for every B fill the MMA warp did not consume.
        const uint64_t t0 = gtimer();
        for (int f = s_consumed[0] + s_consumed[1]; f < issued; ++f) {
          if (blockIdx.x == 0 && f == a.skip_fill) continue;
          const int s = f % kStages;
          const uint32_t par = (f / kStages) & 1;
          while (!mbar_test(bar(FULL + s), par) && gtimer() - t0 < a.drain_ns) {
          }
        }
      }
    }
  } else if (warp == 1 || warp == kIssuer2) {
    // ---------------- MMA issuers ----------------
    // Issuer `me` takes the row tiles whose index (counted over all of this CTA's units) has
    // parity me: those of accumulator slot me.
    static_assert(kAcc == 2, "one issuer per accumulator slot");
    const int me = warp == 1 ? 0 : 1;
    if (lane == 0 && leader) {  // in a pair, the leader issues for both CTAs
      const int accb = me;
      uint32_t a_phase = 0;
      int consumed = 0, g = 0;
      for (int u = worker; u < a.total_units && !*abort_flag; u += workers) {
        int qgroup, chunk;
        unit_coords(a, u, qgroup, chunk);
        const int64_t r0 = static_cast<int64_t>(chunk) * a.chunk_rows;
        const int64_t r1 = min(a.nrows, r0 + a.chunk_rows);
        const int ntiles = static_cast<int>((r1 - r0 + kN - 1) / kN);
        if (!wait(bar(A_FULL), a_phase, abort_flag)) break;
        a_phase ^= 1;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem_a);
        bool ok = true;
        for (int t = (g & 1) == me ? 0 : 1; t < ntiles && ok; t += 2) {
          const int gt = g + t;
          const int stage = gt % kStages;
          ok = wait(bar(FULL + stage), (gt / kStages) & 1, abort_flag);
          if (!ok) break;
          s_consumed[me] = ++consumed;
          tc_fence_after();
          const uint32_t b_addr = smem_u32(smem_b + stage * kAtoms * kBAtomBytes);
          const uint32_t d_base = tmem_base + static_cast<uint32_t>(accb * kTiles * kN);
          if (kAtoms == 1) {
            switch (a.ksteps) {
              case 1: issue_tile<1, 1, kPair>(d_base, a_addr, b_addr); break;
              case 2: issue_tile<1, 2, kPair>(d_base, a_addr, b_addr); break;
              case 3: issue_tile<1, 3, kPair>(d_base, a_addr, b_addr); break;
              default: issue_tile<1, 4, kPair>(d_base, a_addr, b_addr); break;
            }
          } else {
            switch (a.ksteps) {
              case 5: issue_tile<kAtoms, 5, kPair>(d_base, a_addr, b_addr); break;
              case 6: issue_tile<kAtoms, 6, kPair>(d_base, a_addr, b_addr); break;
              case 7: issue_tile<kAtoms, 7, kPair>(d_base, a_addr, b_addr); break;
              default: issue_tile<kAtoms, 8, kPair>(d_base, a_addr, b_addr); break;
            }
          }
          commit_both(EMPTY + stage);
          commit_both(ACC_FULL + accb);
        }
        if (!ok) break;
        g += ntiles;
        commit_both(A_EMPTY);  // A_EMPTY completes once both issuers are done with the unit
      }
      if (*abort_flag) {
        // Wait (bounded) for this issuer's MMAs in flight before the accumulators are freed.
        if (kPair)
          umma_commit_pair_mc(bar(DRAIN + me), 0x1);
        else
          umma_commit(bar(DRAIN + me));
        const uint64_t t0 = gtimer();
        while (!mbar_test(bar(DRAIN + me), 0) && gtimer() - t0 < a.drain_ns) {
        }
      }
    }
  } else if (warp < kIssuer2) {
    // ---------------- epilogue: thread = query ----------------
    // Each query keeps a candidate list of kCap (distance, group) entries in shared memory
    // (sorted best-kKK prefix + entries appended since). Per 64 columns: one three-input
    // max/min tree gives the best score of each 8-row group and of all 64; the warp skips the 64
    // columns when no lane can improve on its threshold (the common case). Otherwise lanes append
    // the groups they can improve on, one entry per group (its best screen distance). When some
    // lane's appends would overflow its list, the warp compacts together first, which tightens
    // every list's threshold to its kKK-th entry: kKK groups, each holding a row at least that
    // close.
    const int quarter = warp & 3;
    const int tile = (warp - 2) >> 2;  // which query tile of the group
    const int qi = quarter * 32 + lane;
    float* bd = buf_d + tile * kM + qi;
    uint32_t* br = buf_r + tile * kM + qi;
    const uint32_t col0 = static_cast<uint32_t>(tile * kN);  // this tile's columns in a slot
    const float kInfF = __int_as_float(0x7f800000);
    int accb = 0;
    int free_stage = kAcc % kStages;  // stage of the tile that next reuses the slot just read
    uint32_t acc_phase = 0;
    // Tiles 0 .. kAcc - 1 (stages 0 .. kAcc - 1) are the first in their slots: nothing to wait for.
    if (lane == 0)
      for (int b = 0; b < kAcc; ++b) arrive_leader(FULL + b);
    for (int u = worker; u < a.total_units; u += workers) {
      int qgroup, chunk;
      unit_coords(a, u, qgroup, chunk);
      const int64_t r0 = static_cast<int64_t>(chunk) * a.chunk_rows;
      const int64_t r1 = min(a.nrows, r0 + a.chunk_rows);
      const int ntiles = static_cast<int>((r1 - r0 + kN - 1) / kN);
      const int q = (first_tile(qgroup) + tile) * kM + qi;
      const bool active = q < a.nq;
      const unsigned* qthr = a.thr_bits + (active ? q : 0);
      float thr = active ? dev::from_ordered_bits(*qthr) : -kInfF;
      const float inv = active ? a.qscale_inv[q] : 0.0f;
      const float qn = (active && kL2) ? a.qnorm2[q] : 0.0f;
      // Start from a prefix of kKK (+inf, ~0) entries; `seen` counts the real entries appended.
#pragma unroll
      for (int i = 0; i < kKK; ++i) {
        bd[i * kLS] = kInfF;
        br[i * kLS] = 0xffffffffu;
      }
      int cnt = kKK, seen = 0;
      bool ok = true;
      // One 64-column half of a tile: rows cb .. cb + 63 (cb a multiple of 64: chunks are
      // multiples of kN rows). best[g]: the best score among elements 8g..8g+7 (max inner product
      // for cosine/IP, min distance for L2); top: the best of all 64.
      auto tree = [&](uint32_t (&r)[64], int64_t cb, float (&best)[8], float& top) {
        float (&v)[64] = *reinterpret_cast<float(*)[64]>(r);  // the loaded bits, used in place
        // Rows past the chunk end and rows the filter rejects take the worst score, so that
        // every group's best is the best of its admitted rows. Only halves that can hold such
        // rows (warp-uniform test) pay for the mask.
        const bool partial = a.bitmap != nullptr || r1 - cb < 64;
        uint64_t admitted = ~0ull;
        if (partial) {
          const int valid = static_cast<int>(r1 - cb < 64 ? r1 - cb : 64);  // rows of this chunk
          admitted = (valid >= 64 ? ~0ull : (valid > 0 ? (1ull << valid) - 1 : 0ull)) &
                     (a.bitmap != nullptr && valid > 0 ? a.bitmap[static_cast<uint64_t>(cb) >> 6]
                                                       : ~0ull);
        }
        if (kL2) {
          // v[j] := ||q||^2 + ||x||^2 - 2<q,x>
          if (!partial) {
#pragma unroll
            for (int j = 0; j < 64; ++j) v[j] = fmaf(-2.0f * inv, v[j], qn + a.xnorm2[cb + j]);
          } else {
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              const bool in = (admitted >> j) & 1ull;
              const float xn = in ? a.xnorm2[cb + j] : 0.0f;
              v[j] = in ? fmaf(-2.0f * inv, v[j], qn + xn) : kInfF;
            }
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
      // Appends the 8-row groups of one half that this lane can improve on. A group enters the
      // candidate list as one entry: its best screen value and its index (rows 8 * index ..
      // 8 * index + 7); the exact re-rank expands it.
      auto screen = [&](const float (&best)[8], float top, int64_t cb) {
        const bool may = active && screen_value<kL2>(top, inv, a.ip_one) <= thr;
        if (!__any_sync(0xffffffffu, may)) return;
        static_assert(kTcGroupRows == 8, "the group tree is built for 8-row groups");
        uint32_t gm = 0;
#pragma unroll
        for (int g = 0; g < 8; ++g)
          gm |= (may && screen_value<kL2>(best[g], inv, a.ip_one) <= thr) ? (1u << g) : 0u;
        // Make room first (all lanes together) when some lane's appends would overflow its
        // list; compaction tightens the threshold, so the groups are tested again.
        if (__any_sync(0xffffffffu, cnt + __popc(gm) > kCap)) {
          compact_buffer<kKK, kAppend>(bd, br, cnt, thr);
          // Publish the tightened bound to the units of other row chunks at once: this unit
          // outputs kKK entries at or below it whatever it appends later.
          if (active) atomicMin(a.thr_bits + q, dev::ordered_bits(thr));
          uint32_t keep = 0;
#pragma unroll
          for (int g = 0; g < 8; ++g)
            keep |= (screen_value<kL2>(best[g], inv, a.ip_one) <= thr) ? (1u << g) : 0u;
          gm &= keep;
        }
        // At most 8 appends and kAppend >= 8 free entries: no further checks. Each entry's
        // position is cnt plus the number of groups before it, so the stores are independent.
        static_assert(kAppend >= 8, "a 64-column group appends up to 8 entries");
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          if ((gm >> g) & 1u) {
            const int pos = cnt + __popc(gm & ((1u << g) - 1u));
            bd[pos * kLS] = screen_value<kL2>(best[g], inv, a.ip_one);
            br[pos * kLS] = static_cast<uint32_t>(cb / kTcGroupRows + g);
          }
        }
        const int np = __popc(gm);
        cnt += np;
        seen += np;
      };
      uint32_t ra[64], rb[64];
      unsigned fresh = ~0u;  // the query's shared threshold, read early and applied later
      for (int t = 0; t < ntiles; ++t) {
        const int64_t row0 = r0 + static_cast<int64_t>(t) * kN;
        if ((t & 7) == 0 && active) fresh = *reinterpret_cast<const volatile unsigned*>(qthr);
        ok = wait(bar(ACC_FULL + accb), acc_phase, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + col0 +
                               static_cast<uint32_t>(accb * kTiles * kN);
        // Both 64-column halves in one round trip; the accumulator goes back to the MMA warp
        // before any screening, so the next MMAs into this slot wait only for the loads.
        static_assert(kN == 128, "the epilogue loads a tile as two 64-column halves");
        tmem_ld64_issue(taddr, ra);
        tmem_ld64_issue(taddr + 64, rb);
        tmem_wait_ld(ra);
        tmem_hold(rb);
        tc_fence_before();
        __syncwarp();
        // The slot is free for the tile kAcc later.
        if (lane == 0) arrive_leader(FULL + free_stage);
        if (++free_stage == kStages) free_stage = 0;
        // Both trees first: the loaded values are dead before any list work (compaction needs
        // the registers).
        float best_a[8], best_b[8], top_a, top_b;
        tree(ra, row0, best_a, top_a);
        tree(rb, row0 + 64, best_b, top_b);
        screen(best_a, top_a, row0);
        screen(best_b, top_b, row0 + 64);
        if (++accb == kAcc) {
          accb = 0;
          acc_phase ^= 1;
        }
        // Tighten with the query's bound from finished units (loaded 7 tiles ago).
        if ((t & 7) == 7) thr = fminf(thr, dev::from_ordered_bits(fresh));
      }
      if (!ok) break;
      compact_buffer<kKK, kAppend>(bd, br, cnt, thr);
      cnt = min(seen, kKK);  // the real entries: they sort before the padding
      if (a.seed_only) {
        // The main launch recomputes these groups bit for bit in the units of the row chunks
        // holding them, and those units together output at least kKK groups at or below this
        // list's kKK-th value: a valid threshold for every unit of the query.
        if (active && cnt == kKK)
          atomicMin(a.thr_bits + q, dev::ordered_bits(bd[(kKK - 1) * kLS]));
      } else if (active) {
        // The whole list, padding included (the finalize reads cand_n entries), as 16-byte
        // stores: a lane's list is contiguous in global memory, strided across lanes.
        const size_t slot = static_cast<size_t>(q) * a.n_chunks + chunk;
        static_assert(kKK % 4 == 0, "lists are written as float4 / uint4");
        float4* cd = reinterpret_cast<float4*>(a.cand_d + slot * kKK);
        uint4* cr = reinterpret_cast<uint4*>(a.cand_r + slot * kKK);
#pragma unroll
        for (int i = 0; i < kKK; i += 4) {
          cd[i / 4] = make_float4(bd[i * kLS], bd[(i + 1) * kLS], bd[(i + 2) * kLS],
                                  bd[(i + 3) * kLS]);
          cr[i / 4] = make_uint4(br[i * kLS], br[(i + 1) * kLS], br[(i + 2) * kLS],
                                 br[(i + 3) * kLS]);
        }
        a.cand_n[slot] = cnt;
        if (cnt == kKK) atomicMin(a.thr_bits + q, dev::ordered_bits(bd[(kKK - 1) * kLS]));
        // Merge this unit's output into the query's running best-kKK list and publish its kKK-th
        // value as the query's threshold: kKK distinct output candidates lie at or below it, which
        // is all a threshold needs. Each unit merges once (its rows are disjoint from every other
        // unit's), under a lock taken with a bounded number of tries: the units of a wave finish
        // together, and a merge skipped after the last try only leaves the bound looser (every
        // later unit of the query then appends more of the groups it sees).
        bool locked = false;
        if (cnt > 0) {
          for (int tries = 0; tries < kMergeTries && !locked; ++tries) {
            locked = atomicCAS(a.glock + q, 0, 1) == 0;
            if (!locked) __nanosleep(64);
          }
        }
        if (locked) {
          __threadfence();
          volatile float* gq = a.gbest + static_cast<size_t>(q) * kMaxKK;
          // Both lists are sorted ascending and padded with +inf to 32, so c[i] = min(g[i],
          // b[31 - i]) holds the 32 smallest of both as a bitonic sequence, which a 32-input
          // bitonic merge (distances only) sorts; its first kKK are the new running list.
          float c[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float gi = i < kKK ? gq[i] : kInfF;
            const float bi = 31 - i < kKK ? bd[(31 - i) * kLS] : kInfF;
            c[i] = fminf(gi, bi);
          }
#pragma unroll
          for (int stride = 16; stride > 0; stride >>= 1) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
              const float x = fminf(c[lo], c[hi]);
              c[hi] = fmaxf(c[lo], c[hi]);
              c[lo] = x;
            }
          }
#pragma unroll
          for (int i = 0; i < kKK; ++i) gq[i] = c[i];
          __threadfence();
          if (c[kKK - 1] < kInfF) atomicMin(a.thr_bits + q, dev::ordered_bits(c[kKK - 1]));
          atomicExch(a.glock + q, 0);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // In a pair, neither CTA frees its tensor memory or leaves while the other may still reach its
  // barriers or the leader's MMAs its memory.
  if (kPair) cluster_sync();
  tc_fence_after();
  if (warp == 1) {
    if (kPair)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(kAcc * kTiles * kN));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(kAcc * kTiles * kN));
  }
}

// The query-wide best lists start at +inf, unlocked.
__global__ void init_best_kernel(float* gbest, size_t n, int* glock, size_t nq) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t i0 = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  for (size_t i = i0; i < n; i += stride) gbest[i] = __int_as_float(0x7f800000);
  for (size_t i = i0; i < nq; i += stride) glock[i] = 0;
}

// ---- fp16 operands ---------------------------------------------------------------------------------

__device__ __forceinline__ float pow2_scale_for(float maxabs) {
  // Keep data in fp16's comfortable range: scale by 2^E only when the largest magnitude is
  // outside [2^-8, 2^14]; the scale is a power of two, so scaling itself is exact.
  if (!(maxabs > 0.0f)) return 1.0f;
  int e;
  frexpf(maxabs, &e);  // maxabs in [2^(e-1), 2^e)
  if (e >= -7 && e <= 14) return 1.0f;
  return ldexpf(1.0f, 13 - e);
}

// Rows -> fp16 (kpad columns, zero padded) with one scale for the whole index (from the max |x|
// in stats[0]); max row error into stats[1].
__global__ void rows_to_f16_kernel(const float* __restrict__ x, size_t n, int dim, int kpad,
                                   __half* __restrict__ out, unsigned* __restrict__ stats) {
  const int lane = threadIdx.x & 31;
  const size_t row = static_cast<size_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n) return;
  unsigned* max_err_bits = stats + 1;
  const float scale = pow2_scale_for(__uint_as_float(stats[0]));
  const float inv = 1.0f / scale;
  double e2 = 0.0;
  for (int c = lane; c < kpad; c += 32) {
    const float v = c < dim ? x[row * dim + c] : 0.0f;
    const __half h = __float2half_rn(v * scale);
    out[row * kpad + c] = h;
    const double diff = static_cast<double>(v) - static_cast<double>(__half2float(h)) * inv;
    e2 += diff * diff;
  }
  for (int o = 16; o > 0; o >>= 1) e2 += __shfl_xor_sync(0xffffffffu, e2, o);
  if (lane == 0) atomicMax(max_err_bits, __float_as_uint(static_cast<float>(sqrt(e2)) * 1.001f + 1e-30f));
}

__global__ void max_abs_kernel(const float* __restrict__ x, size_t total, unsigned* out_bits) {
  float m = 0.0f;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    m = fmaxf(m, fabsf(x[i]));
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));
}

// Queries (already normalized rows of qp, stride dpad) -> fp16 with a per-query power-of-two
// scale; 1/(s_q s_x); and the screen's error bound eps[q] against the reference's distance. Rows
// nq .. nq_pad - 1 of q16 (padding up to whole query tiles) are zeroed. x_stats: the fp16 copy's
// words (max |x|, max row error).
__global__ void queries_to_f16_kernel(const float* __restrict__ qp, int nq, int nq_pad, int dim,
                                      int dpad, int kpad, const unsigned* __restrict__ x_stats,
                                      float x_max_norm, bool l2, bool drop_qnorm, float gamma,
                                      __half* __restrict__ q16, float* __restrict__ qscale_inv,
                                      float* __restrict__ qnorm2, float* __restrict__ eps) {
  const int lane = threadIdx.x & 31;
  const int q = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (q >= nq_pad) return;
  if (q >= nq) {
    for (int c = lane; c < kpad; c += 32) q16[static_cast<size_t>(q) * kpad + c] = __float2half_rn(0.0f);
    return;
  }
  const float x_scale = pow2_scale_for(__uint_as_float(x_stats[0]));
  const float x_err = __uint_as_float(x_stats[1]);
  const float* v = qp + static_cast<size_t>(q) * dpad;
  float mx = 0.0f;
  for (int c = lane; c < dim; c += 32) mx = fmaxf(mx, fabsf(v[c]));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float s = pow2_scale_for(mx);
  const float inv_s = 1.0f / s;
  double e2 = 0.0, n2 = 0.0;
  for (int c = lane; c < kpad; c += 32) {
    const float x = c < dim ? v[c] : 0.0f;
    const __half h = __float2half_rn(x * s);
    q16[static_cast<size_t>(q) * kpad + c] = h;
    const double diff = static_cast<double>(x) - static_cast<double>(__half2float(h)) * inv_s;
    e2 += diff * diff;
    n2 += static_cast<double>(x) * x;
  }
  for (int o = 16; o > 0; o >>= 1) {
    e2 += __shfl_xor_sync(0xffffffffu, e2, o);
    n2 += __shfl_xor_sync(0xffffffffu, n2, o);
  }
  if (lane == 0) {
    const double eq = sqrt(e2) * 1.001, qn = sqrt(n2) * 1.001;
    const double xm = static_cast<double>(x_max_norm), ex = static_cast<double>(x_err);
    const double u = 5.9604644775390625e-08;  // 2^-24
    // |<q,x> - <q16,x16>| <= eq*||x|| + ||q16||*ex, plus float32 accumulation in the tensor core
    // and the reference's own float32 summation (gamma each, relative to sum |q_i x_i|).
    const double dot_err = eq * xm + (qn + eq) * ex + 2.0 * gamma * (qn + eq) * (xm + ex);
    double e;
    if (l2) {
      const double s2 = (qn + xm) * (qn + xm);
      e = 2.0 * dot_err + 3.0 * gamma * s2 + 4.0 * u * s2;
    } else {
      e = dot_err + 4.0 * u * (1.0 + qn * xm);
    }
    eps[q] = static_cast<float>(e * 1.01 + 1e-30);
    qscale_inv[q] = 1.0f / (s * x_scale);
    qnorm2[q] = drop_qnorm ? 0.0f : static_cast<float>(n2);
  }
}

// ---- tensor maps ---------------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (fn == nullptr) fail(QV_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  return fn;
}

uint64_t drain_limit_ns() {
  // Copies and MMAs in flight finish within microseconds; 10 ms, or the wait bound if longer.
  const uint64_t wait_ns = static_cast<uint64_t>(wait_limit_cycles() / 2);
  return std::min<uint64_t>(kTimeoutNs, std::max<uint64_t>(10000000ull, wait_ns));
}

int test_skip_fill() {
  const char* e = std::getenv("QV_TC_TEST_SKIP_FILL");
  return (e == nullptr || *e == '\0') ? -1 : std::atoi(e);
}

long long wait_limit_cycles() {
  const char* e = std::getenv("QV_TC_WAIT_LIMIT_US");
  if (e == nullptr || *e == '\0') return kTimeoutCycles;
  const long long us = std::atoll(e);
  return us > 0 ? us * 2000 : kTimeoutCycles;
}

// 2-D fp16 tensor [rows][kpad], boxes of 64 columns x box_rows rows, 128-byte swizzle, zero fill.
CUtensorMap make_map(const void* base, uint64_t rows, uint64_t kpad, uint32_t box_rows) {
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t dims[2] = {kpad, rows};
  const cuuint64_t strides[1] = {kpad * sizeof(__half)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kAtomK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base),
                                 dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(QV_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return m;
}

}  // namespace tc

// ---- host side ------------------------------------------------------------------------------------

// The narrow screen (this file) takes dim <= 128 and k <= 24; the wide screen (flat_tc_wide.cu)
// dim <= 768 and k <= 204.
bool flat_tc_is_wide(const FlatState& s, size_t k) {
  return s.dim > 128 || k + 8 > static_cast<size_t>(tc::kMaxKK);
}

bool flat_tc_eligible(const FlatState& s, size_t k) {
  const char* e = std::getenv("QV_FLAT_SCREEN");
  if (e != nullptr && std::strcmp(e, "simt") == 0) return false;
  if (s.n < static_cast<size_t>(tc::kN)) return false;
  return flat_tc_is_wide(s, k) ? flat_tc_wide_fits(s, k) : true;
}

// The narrow screen runs in single CTAs unless QV_TC_PAIR=1 selects CTA pairs (tcgen05
// cta_group::2); both give identical results. On config 1 (1,183,514 x 100 cosine, 10,000
// queries) pairs took 3.20 ms against 2.18 ms: with the epilogue's work switched off the pair's
// copy and MMA pipeline alone took 2.16 ms against 1.60 ms, and 1.82 ms even without MMAs, so
// the cross-CTA barrier hand-offs per row tile, not shared-memory bandwidth, set its pace.
bool flat_tc_pair(const FlatState& s, size_t k) {
  if (flat_tc_is_wide(s, k)) return false;
  const char* e = std::getenv("QV_TC_PAIR");
  if (e == nullptr || e[0] != '1') return false;
  return sm_count(s.device) >= 2;
}

// Queries per work unit's query group and the number of concurrent workers (CTAs, or pairs).
int flat_tc_group_rows(const FlatState& s, size_t k) {
  if (flat_tc_is_wide(s, k)) return tc::kM;
  return (flat_tc_pair(s, k) ? 2 : 1) * tc::kTiles * tc::kM;
}
int flat_tc_workers(const FlatState& s, size_t k) {
  return flat_tc_pair(s, k) ? sm_count(s.device) / 2 : sm_count(s.device);
}

// Best-list length: k + 8 groups or more (the certificate's margin); 24 when that suffices,
// which tightens thresholds and shortens the finalize's re-rank; the wide screen rounds k + 8 up
// to a multiple of 16 (its lists are merged in 16-entry chunks).
int flat_tc_kk(const FlatState& s, size_t k) {
  if (flat_tc_is_wide(s, k)) return flat_tc_wide_kk(k);
  return k + 8 <= 24 ? 24 : tc::kMaxKK;
}

// Builds (once per set of rows) the fp16 copy of the index and its error statistics, entirely on
// the device: nothing here waits for the GPU. Searches on other streams wait for the copy through
// the x16_ready event.
void flat_tc_prepare(FlatState& s, cudaStream_t st) {
  if (s.x16.bytes() != 0 && s.x16_rows == s.n) {
    QV_CUDA(cudaStreamWaitEvent(st, s.x16_ready, 0));
    return;
  }
  // At least one full 64-column swizzle atom, so a TMA box never extends past a row.
  const int kpad = static_cast<int>(std::max<size_t>(64, ceil_div(s.dim, 16) * 16));
  if (s.x16_ready == nullptr) QV_CUDA(cudaEventCreateWithFlags(&s.x16_ready, cudaEventDisableTiming));
  if (s.x16_stats.bytes() == 0) s.x16_stats.allocate(2 * sizeof(unsigned));
  s.x16.allocate(s.n * kpad * sizeof(__half));
  QV_CUDA(cudaMemsetAsync(s.x16_stats.get(), 0, 2 * sizeof(unsigned), st));
  tc::max_abs_kernel<<<std::min<size_t>(ceil_div(s.n * s.dim, 256), 4096), 256, 0, st>>>(
      s.x.get<float>(), s.n * s.dim, s.x16_stats.get<unsigned>());
  check_launch("max_abs_kernel");
  tc::rows_to_f16_kernel<<<ceil_div(s.n, 8), 256, 0, st>>>(s.x.get<float>(), s.n,
                                                          static_cast<int>(s.dim), kpad,
                                                          s.x16.get<__half>(),
                                                          s.x16_stats.get<unsigned>());
  check_launch("rows_to_f16_kernel");
  QV_CUDA(cudaEventRecord(s.x16_ready, st));
  s.kpad = static_cast<size_t>(kpad);
  s.x16_rows = s.n;
}

// Scratch layout of one tensor-core screen (offsets into the block flat_tc_scratch_bytes sizes).
struct TcScratch {
  size_t q16, qinv, qn2, gbest, glock, lists, total;
};
// group_rows: queries per unit's group (the fp16 queries are padded to whole groups, so that no
// TMA box extends past the tensor).
static TcScratch tc_scratch_layout(size_t kpad, size_t nq, int kk, size_t list_bytes,
                                   size_t group_rows) {
  const size_t nq_pad = ceil_div(nq, group_rows) * group_rows;
  TcScratch L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = (off + bytes + 255) & ~size_t{255};
    return at;
  };
  L.q16 = take(nq_pad * kpad * sizeof(__half));
  L.qinv = take(nq * sizeof(float));
  L.qn2 = take(nq * sizeof(float));
  L.gbest = take(nq * static_cast<size_t>(std::max(kk, tc::kMaxKK)) * sizeof(float));
  L.glock = take(nq * sizeof(int));
  L.lists = take(list_bytes);
  L.total = off;
  return L;
}

// The wide screen's per-CTA working lists (none for the narrow screen, whose lists live in
// shared memory).
static size_t tc_list_bytes(const FlatState& s, int kk) {
  return kk > tc::kMaxKK || s.dim > 128 ? flat_tc_wide_list_bytes(s, kk) : 0;
}

size_t flat_tc_scratch_bytes(const FlatState& s, size_t nq, size_t k, int kk) {
  const size_t kpad = std::max<size_t>(64, ceil_div(s.dim, 16) * 16);
  return tc_scratch_layout(kpad, nq, kk, tc_list_bytes(s, kk),
                           static_cast<size_t>(std::max(flat_tc_group_rows(s, k), 2 * tc::kM)))
      .total;
}

// Runs the tensor-core screen for the queries in qp (normalized, dpad stride). Writes the per-query
// candidates in the layout flat_finalize_kernel reads, and eps[q].
void flat_screen_tc(const FlatState& s, const float* qp, int dpad, size_t nq, size_t k,
                    const uint64_t* d_bitmap, int n_chunks, int64_t chunk_rows, int kk,
                    float* cand_d, uint32_t* cand_r, int* cand_n, unsigned* thr_bits, float* eps,
                    int* err, void* scratch, cudaStream_t st) {
  const bool wide = kk > tc::kMaxKK || s.dim > 128;
  QV_REQUIRE(wide || kk == 24 || kk == tc::kMaxKK,
             "tensor-core screen: unsupported best-list length");
  const int kpad = static_cast<int>(s.kpad);
  const bool l2 = s.metric == QV_METRIC_L2;
  const bool pair = !wide && flat_tc_pair(s, k);
  // Whole query groups (zero rows past nq), so no TMA box extends past the tensor; the scratch
  // pads to at least two query tiles for every screen.
  const size_t group_rows =
      static_cast<size_t>(std::max(flat_tc_group_rows(s, k), 2 * tc::kM));
  const size_t nq_pad = ceil_div(nq, group_rows) * group_rows;
  const TcScratch L = tc_scratch_layout(s.kpad, nq, kk, tc_list_bytes(s, kk), group_rows);
  unsigned char* base = static_cast<unsigned char*>(scratch);
  __half* q16 = reinterpret_cast<__half*>(base + L.q16);
  float* qinv = reinterpret_cast<float*>(base + L.qinv);
  float* qn2 = reinterpret_cast<float*>(base + L.qn2);
  float* gbest = reinterpret_cast<float*>(base + L.gbest);
  int* glock = reinterpret_cast<int*>(base + L.glock);
  const double gamma = (kpad + 2) * std::ldexp(1.0, -23);
  tc::queries_to_f16_kernel<<<ceil_div(nq_pad, 8), 256, 0, st>>>(
      qp, static_cast<int>(nq), static_cast<int>(nq_pad), static_cast<int>(s.dim), dpad, kpad,
      s.x16_stats.get<unsigned>(), s.max_norm, l2, s.drop_qnorm, static_cast<float>(gamma), q16,
      qinv, qn2, eps);
  check_launch("queries_to_f16_kernel");
  if (wide) {
    const CUtensorMap mq = tc::make_map(q16, nq_pad, kpad);
    flat_screen_tc_wide(s, qp, dpad, nq, d_bitmap, n_chunks, chunk_rows, kk, cand_d, cand_r,
                        cand_n, thr_bits, eps, err, mq, q16, qinv, qn2, base + L.lists, st);
    return;
  }
  tc::init_best_kernel<<<static_cast<unsigned>(
                             std::min<size_t>(ceil_div(nq * tc::kMaxKK, 256), 1024)),
                         256, 0, st>>>(gbest, nq * tc::kMaxKK, glock, nq);
  check_launch("init_best_kernel");
  const CUtensorMap mq = tc::make_map(q16, nq_pad, kpad);
  // A pair's CTAs each load 64 rows of every 128-row tile.
  const CUtensorMap mx = tc::make_map(s.x16.get(), s.n, kpad, pair ? tc::kN / 2 : tc::kN);
  tc::Args a{};
  a.nq = static_cast<int>(nq);
  a.n_qgroups = static_cast<int>(ceil_div(nq, static_cast<size_t>(flat_tc_group_rows(s, k))));
  a.n_chunks = n_chunks;
  a.total_units = a.n_qgroups * n_chunks;
  // K steps of 16 elements cover the dimension; the zero padding beyond the last one (up to the
  // 64-element atom) adds nothing to the products and is not multiplied.
  a.ksteps = static_cast<int>(ceil_div(static_cast<size_t>(s.dim), 16));
  a.nrows = static_cast<int64_t>(s.n);
  a.chunk_rows = chunk_rows;
  a.l2 = l2;
  a.qscale_inv = qinv;
  a.qnorm2 = qn2;
  a.xnorm2 = s.xnorm2.get<float>();
  a.bitmap = d_bitmap;
  a.cand_d = cand_d;
  a.cand_r = cand_r;
  a.cand_n = cand_n;
  a.thr_bits = thr_bits;
  // Unit order: QV_FLAT_TC_ORDER=q selects query-tile-major (all row chunks of a query tile run
  // together, sharing thresholds); the default row-chunk-major order shares row chunks in L2.
  const char* order = std::getenv("QV_FLAT_TC_ORDER");
  a.qmajor = order != nullptr && order[0] == 'q';
  a.gbest = gbest;
  a.glock = glock;
  a.err = err;
  a.wait_cycles = tc::wait_limit_cycles();
  a.drain_ns = tc::drain_limit_ns();
  a.skip_fill = tc::test_skip_fill();
  a.ip_one = s.neg_ip ? 0.0f : 1.0f;
  a.seed_only = false;
  const int atoms = kpad > tc::kAtomK ? 2 : 1;
  const int max_workers = flat_tc_workers(s, k);
  const int workers = std::min(a.total_units, max_workers);
  const int grid = pair ? 2 * workers : workers;
  // Threshold seeding (QV_TC_SEED=1): in the main launch's first wave every query has several
  // units running at once, all starting from an infinite threshold. A short first launch over a
  // few 4096-row sub-chunks (as many per query group as fill the GPU, together at most an eighth
  // of the rows) publishes each query's kKK-th best group there as its starting threshold. Off
  // by default: on config 1 the screen took 2.25 ms with it against 2.19 ms without, so the
  // first wave's appends are not what the candidate work costs.
  constexpr int64_t kSeedRows = 4096;
  tc::Args seed = a;
  const char* seed_env = std::getenv("QV_TC_SEED");
  const int seed_chunks = static_cast<int>(std::min<int64_t>(
      std::max(1, max_workers / std::max(1, a.n_qgroups)),
      static_cast<int64_t>(s.n) / (8 * kSeedRows)));
  const bool seeding = n_chunks > 1 && seed_chunks >= 1 && seed_env != nullptr &&
                       seed_env[0] == '1';
  if (seeding) {
    seed.seed_only = true;
    seed.skip_fill = -1;
    seed.n_chunks = seed_chunks;
    seed.chunk_rows = kSeedRows;
    seed.nrows = kSeedRows * seed_chunks;
    seed.total_units = a.n_qgroups * seed_chunks;
  }
  const int seed_workers = std::min(seed.total_units, max_workers);
  KernelTimer timer(st, "flat_screen_tc_kernel", 2.0 * nq * static_cast<double>(s.n) * s.dim,
                    false);
  // Shared memory of one instantiation: alignment slack, the query tiles, the row ring, the
  // candidate lists and the barriers.
  auto smem_of = [&](auto ring, int at) {
    using R = decltype(ring);
    const size_t b_atom = pair ? tc::kAtomBytes / 2 : tc::kAtomBytes;
    return 1024 + static_cast<size_t>(at) * tc::kAtomBytes * tc::kTiles +
           static_cast<size_t>(R::kStages) * at * b_atom +
           static_cast<size_t>(kk + R::kAppend) * tc::kLS * 8 + (2 * R::kStages + tc::kAcc + 4) * 8;
  };
  auto launch = [&](auto kernel, size_t smem, const tc::Args& args, int grid_) {
    QV_REQUIRE(smem <= 227 * 1024, "tensor-core screen: shared memory layout too large");
    QV_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (!pair) {
      kernel<<<grid_, tc::kThreads, smem, st>>>(mq, mx, args);
      return;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid_));
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QV_CUDA(cudaLaunchKernelEx(&cfg, kernel, mq, mx, args));
  };
  // One instantiation per (atoms, metric, best-list length, pair).
  auto pick = [&](auto atoms_c, auto kk_c, auto pair_c) {
    constexpr int kA = decltype(atoms_c)::value, kK = decltype(kk_c)::value;
    constexpr bool kP = decltype(pair_c)::value;
    const size_t smem = smem_of(tc::Ring<kK, kP, kA>{}, kA);
    auto kernel = l2 ? tc::flat_screen_tc_kernel<kA, true, kK, kP>
                     : tc::flat_screen_tc_kernel<kA, false, kK, kP>;
    if (seeding) launch(kernel, smem, seed, pair ? 2 * seed_workers : seed_workers);
    launch(kernel, smem, a, grid);
  };
  using A1 = std::integral_constant<int, 1>;
  using A2 = std::integral_constant<int, 2>;
  using K24 = std::integral_constant<int, 24>;
  using K32 = std::integral_constant<int, 32>;
  using P0 = std::false_type;
  using P1 = std::true_type;
  if (atoms == 2) {
    if (kk == 24)
      pair ? pick(A2{}, K24{}, P1{}) : pick(A2{}, K24{}, P0{});
    else
      pair ? pick(A2{}, K32{}, P1{}) : pick(A2{}, K32{}, P0{});
  } else {
    if (kk == 24)
      pair ? pick(A1{}, K24{}, P1{}) : pick(A1{}, K24{}, P0{});
    else
      pair ? pick(A1{}, K32{}, P1{}) : pick(A1{}, K32{}, P0{});
  }
  timer.stop();
  check_launch("flat_screen_tc_kernel");
  // A barrier timeout is reported through *err: the finalize then sends every query to the exact
  // rescan and counts the timeout in the search's report words.
}

}  // namespace qv
