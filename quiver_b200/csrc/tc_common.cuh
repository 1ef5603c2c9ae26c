// tcgen05 / TMA / mbarrier building blocks shared by the tensor-core screens (flat_tc.cu,
// flat_tc_wide.cu): inline-PTX wrappers for sm_100a, the fp16 MMA instruction descriptor, the
// bounded barrier wait, and the epilogue's group reductions and compare-exchange.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "qv_state.h"

namespace qv {
namespace tc {

constexpr int kM = 128;          // queries per unit = TMEM lanes
constexpr int kN = 128;          // database rows per MMA tile
constexpr int kAtomK = 64;       // fp16 elements per 128-byte swizzled row
constexpr int kAtomBytes = 128 * 128;  // one 128-row x 128-byte swizzle atom column
constexpr uint64_t kTimeoutNs = 2000000000ull;       // drain bound (global timer)
constexpr long long kTimeoutCycles = 4000000000ll;     // default wait bound: ~2 s at 2 GHz
constexpr uint32_t kSuspendHintNs = 100000;           // one sleeping try_wait: at most 0.1 ms
constexpr uint32_t kIdesc = (1u << 4)            // D format f32
                            | (0u << 7)          // A f16
                            | (0u << 10)         // B f16
                            | ((kN >> 3) << 17)  // N
                            | ((kM >> 4) << 24); // M

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: a waiting thread sleeps in hardware until the phase
// completes (or the hint elapses) instead of spinning, so waiting warps leave the scheduler's
// issue slots to the warps that share it.
__device__ __forceinline__ bool mbar_sleep_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of `parity` to complete. False on timeout or abort. Each try sleeps
// at most kSuspendHintNs; the bound (limit, in SM clock cycles: clock64 is a cheap per-SM counter,
// the global timer a slow read) is a kernel argument, ~2 s by default. On timeout the wait raises
// the CTA's abort flag and the launch's error word, so that every other wait of the CTA returns.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, long long limit) {
  if (mbar_test(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_sleep_test(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      atomicExch(err, 1);
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// K-major, 128-byte swizzle (8-row groups 1024 bytes apart), sm_100 descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return (static_cast<uint64_t>(addr >> 4) & 0x3FFFull) | (1ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc)
      : "memory");
}
// The same MMA with A read from tensor memory: a_tmem addresses the first 32-bit column of the
// K step (lane = row of A, two consecutive fp16 K elements per column, the lower one in the low
// half), B from shared memory as above.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(kIdesc), "r"(acc)
      : "memory");
}
// Stores 32 consecutive 32-bit columns of this thread's TMEM lane (the warp's 32 lanes at once).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Starts a 64-column TMEM load (32 lanes x 64 columns, one value per column for this thread's
// lane); the registers are valid only after tmem_wait_ld.
__device__ __forceinline__ void tmem_ld64_issue(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
}
// Waits for this thread's TMEM loads. The registers of the load being waited for pass through
// the statement, so that no use of them is scheduled above the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[64]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]), "+r"(r[32]), "+r"(r[33]), "+r"(r[34]), "+r"(r[35]), "+r"(r[36]), "+r"(r[37]), "+r"(r[38]), "+r"(r[39]), "+r"(r[40]), "+r"(r[41]), "+r"(r[42]), "+r"(r[43]), "+r"(r[44]), "+r"(r[45]), "+r"(r[46]), "+r"(r[47]), "+r"(r[48]), "+r"(r[49]), "+r"(r[50]), "+r"(r[51]), "+r"(r[52]), "+r"(r[53]), "+r"(r[54]), "+r"(r[55]), "+r"(r[56]), "+r"(r[57]), "+r"(r[58]), "+r"(r[59]), "+r"(r[60]), "+r"(r[61]), "+r"(r[62]), "+r"(r[63])
               :
               : "memory");
}
// Orders every later use of r after the preceding tmem_wait_ld (for a second load waited for
// by the same wait).
__device__ __forceinline__ void tmem_hold(uint32_t (&r)[64]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]), "+r"(r[32]), "+r"(r[33]), "+r"(r[34]), "+r"(r[35]), "+r"(r[36]), "+r"(r[37]), "+r"(r[38]), "+r"(r[39]), "+r"(r[40]), "+r"(r[41]), "+r"(r[42]), "+r"(r[43]), "+r"(r[44]), "+r"(r[45]), "+r"(r[46]), "+r"(r[47]), "+r"(r[48]), "+r"(r[49]), "+r"(r[50]), "+r"(r[51]), "+r"(r[52]), "+r"(r[53]), "+r"(r[54]), "+r"(r[55]), "+r"(r[56]), "+r"(r[57]), "+r"(r[58]), "+r"(r[59]), "+r"(r[60]), "+r"(r[61]), "+r"(r[62]), "+r"(r[63])
               :
               : "memory");
}
// Screen distance of one accumulator element: for L2 the element already is the distance; for
// cosine / inner product it is the raw (scaled) inner product and the distance is
// one - dot * inv (one = 1, or 0 where inner-product distances are -<q,x>).
// fmaf rounds once and is monotone in the element, so the best raw value gives the best distance.
template <bool kL2>
__device__ __forceinline__ float screen_value(float x, float inv, float one) {
  return kL2 ? x : fmaf(-x, inv, one);
}

// Three-input max / min (one PTX instruction on sm_100a).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float min3f(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <bool kMax>
__device__ __forceinline__ float best2(float a, float b) {
  return kMax ? fmaxf(a, b) : fminf(a, b);
}
template <bool kMax>
__device__ __forceinline__ float best3(float a, float b, float c) {
  return kMax ? max3f(a, b, c) : min3f(a, b, c);
}

// best[g] = best of v[8g .. 8g+7] (max when kMax, else min), top = best of all 64, with
// three-input operations: 4 per 8-element group and 4 for the top (36 in all, depth 3 + 3).
template <bool kMax>
__device__ __forceinline__ void group_best8(const float (&v)[64], float (&best)[8], float& top) {
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const float* e = v + 8 * g;
    const float x = best3<kMax>(e[0], e[1], e[2]);
    const float y = best3<kMax>(e[3], e[4], e[5]);
    best[g] = best3<kMax>(x, y, best2<kMax>(e[6], e[7]));
  }
  const float x = best3<kMax>(best[0], best[1], best[2]);
  const float y = best3<kMax>(best[3], best[4], best[5]);
  top = best3<kMax>(x, y, best2<kMax>(best[6], best[7]));
}

// Per-lane candidate lists: entry i of list l lives at i * kLS + l (the lanes of a warp hold
// adjacent lists, so their accesses never share a bank). A list is a sorted prefix of exactly
// KK entries (padded with (+inf, ~0) at the start of a work unit) followed by up to kAppend
// entries appended since (kCap = KK + kAppend in all; Ring<KK>::kAppend).

// Compare-exchange of two (distance, group) entries in registers: afterwards (da, ra) is the
// smaller in (distance, group) order.
__device__ __forceinline__ void cex(float& da, uint32_t& ra, float& db, uint32_t& rb) {
  const bool sw = dev::key_less(db, rb, da, ra);
  const float td = sw ? db : da;
  const uint32_t tr = sw ? rb : ra;
  db = sw ? da : db;
  rb = sw ? ra : rb;
  da = td;
  ra = tr;
}

// Bound of the screens' mbarrier waits in SM clock cycles: QV_TC_WAIT_LIMIT_US microseconds
// (counted at 2 GHz) when set, else kTimeoutCycles (~2 s). A short bound lets a test make a wait
// run out and check that the search reports it and the context stays usable.
long long wait_limit_cycles();
// Bound of the abort path's waits for copies and MMAs in flight (global-timer nanoseconds).
uint64_t drain_limit_ns();
// Failure-detection test hook: QV_TC_TEST_SKIP_FILL=n makes CTA 0's producer skip its n-th ring
// fill (no copy, no arrival), so that a barrier wait runs out and the abort path is exercised;
// -1 (unset) in normal use.
int test_skip_fill();

// ---- CTA pairs (cluster of two CTAs, tcgen05 cta_group::2) ----------------------------------------
// In a pair, the even CTA (rank 0) issues MMAs of M = 256 rows: each CTA holds its own 128 rows
// of A and half of B's N rows, and its own half of D in its TMEM. Barriers the pair shares live
// in the leader's shared memory; the peer reaches them through shared::cluster addresses.
constexpr uint32_t kIdescPair = (1u << 4)               // D format f32
                                | ((kN >> 3) << 17)     // N = 128 (64 rows from each CTA)
                                | ((2 * kM >> 4) << 24);  // M = 256 (128 rows from each CTA)

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of `addr` (a shared::cta address of this CTA) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Arrive on a barrier of the pair (a shared::cluster address), releasing at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx_cluster(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
// try_wait acquiring at cluster scope (the barrier's arrivals may come from the peer CTA).
__device__ __forceinline__ bool mbar_test_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// The same with a suspend-time hint: a waiting thread sleeps in hardware until the phase completes
// (or the hint elapses) instead of spinning, leaving issue slots to the warps that share it.
__device__ __forceinline__ bool mbar_sleep_test_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity,
                                                  volatile int* abort_flag, int* err,
                                                  long long limit) {
  if (mbar_test_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  for (;;) {
    if (mbar_sleep_test_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      atomicExch(err, 1);
      return false;
    }
  }
}
// TMA load into this CTA's shared memory whose completion is counted on a barrier of the pair
// (cluster_bar: a shared::cluster address, the leader's barrier). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(cluster_bar)
      : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a, uint64_t b,
                                              uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdescPair), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                                 uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(kIdescPair), "r"(acc)
      : "memory");
}
// Arrives on the barrier at offset `bar` in every CTA of `mask` once the pair's MMAs issued so
// far have completed.
__device__ __forceinline__ void umma_commit_pair_mc(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

// Tensor maps (host): 2-D fp16 tensor [rows][kpad], boxes of 64 columns x 128 rows, 128-byte
// swizzle, zero fill past the tensor's edges.
CUtensorMap make_map(const void* base, uint64_t rows, uint64_t kpad, uint32_t box_rows = kM);

}  // namespace tc

// The wide screen (flat_tc_wide.cu): rows up to 768 columns, best lists up to 128 groups. mq is
// the queries' tensor map; qinv / qn2 as the screen in flat_tc.cu computes them; lists is
// flat_tc_wide_list_bytes of scratch.
void flat_screen_tc_wide(const FlatState& s, const float* qp, int dpad, size_t nq,
                         const uint64_t* d_bitmap, int n_chunks, int64_t chunk_rows, int kk,
                         float* cand_d, uint32_t* cand_r, int* cand_n, unsigned* thr_bits,
                         float* eps, int* err, const CUtensorMap& mq, const __half* q16,
                         const float* qinv, const float* qn2, void* lists, cudaStream_t st);
}  // namespace qv
