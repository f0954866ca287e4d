// fa_kernel.cuh -- the sm_100a warp-specialised flash-attention forward.
//
// Operator (reference semantics: backends/npu_fa/backend.py:36-49, FP32
// formula backends/expert_v2/impl_tl.py:701-717):
//   O[b,h] = softmax(Q[b,h] K[b,kv]^T * scale) V[b,kv],  kv = b*Hkv + h/(Hq/Hkv)
// (GQA head map of panel_kernel.h:274), non-causal, D = 128, FP16 in/out.
//
// Work decomposition.  A work unit is one 128-row query block of one (b, hq),
// linearised ((b*Hq)+hq)*ceil(Nq/128)+qb (cce_task.h:28-35 order).  A work
// item is two consecutive units of the same head (256 query rows) that share
// every K/V tile; a lone trailing unit is processed as a pair whose second
// tile repeats the first one's rows and is not stored.  Items are dealt
// round-robin to a persistent grid of one CTA per SM.
//
// CTA roles (384 threads = 3 warpgroups):
//   warps 0-3   softmax warpgroup 0: query tile 0 (TMEM lanes = rows)
//   warps 4-7   softmax warpgroup 1: query tile 1
//   warp  8     MMA issuer (one thread): tcgen05.mma for QK^T and PV
//   warp  9     TMA producer (one thread): Q tiles and the K/V ring
//   warps 10-11 idle (complete warpgroup 2 for the register split)
//
// Tensor memory (512 columns x 128 lanes x 32 bit):
//   [  0,128) S0 = Q0 K^T (FP32); its first 64 columns are reused for P0
//             (FP16 pairs) once the softmax has read S0
//   [128,256) S1 / P1
//   [256,384) O0 accumulator (FP32)
//   [384,512) O1 accumulator (FP32)
//
// Shared memory (1024-B aligned; every tile = two 64-column halves of
// 128 rows x 128 B in the 128-byte swizzle the TMA writes):
//   Q0, Q1 (2 x 32 KiB; each also stages its tile's FP16 output for the TMA
//   store), K/V ring (kStages x 32 KiB; K_j and V_j take alternate slots),
//   mbarriers, TMEM base address, abort flag.
//
// Per KV block j the MMA thread issues, in this order,
//   PV0(j-1) .. S0(j) .. PV1(j-1) .. S1(j)
// so that the softmax of one tile overlaps the tensor-core work of the other.
// S_t(j+1) overwrites the columns PV_t(j) reads P_t from; both are issued by
// the same thread in that order and the tensor pipe executes them in order.
//
// Online softmax (per query row, one thread per row): running reference
// maximum m (log2 domain), running sum l.  The reference maximum moves only
// when a block's maximum exceeds it by more than kRescaleLog2 (lazy
// rescaling), so P <= 2^kRescaleLog2 and O/l is exact at the end whatever the
// reference.  When it moves, the warp rescales its 32 rows of O in TMEM.
//
// Every wait is bounded (global timer); on expiry the kernel records
// B200FA_DEV_TIMEOUT in the workspace, every role leaves its loop, in-flight
// copies and MMAs are drained with a second bound, TMEM is freed and the
// kernel returns.
#pragma once
#include <cstdint>
#include <cuda.h>
#include "ptx.cuh"

namespace b200fa {

constexpr int kBlockM = 128;    // query rows per tile
constexpr int kBlockN = 128;    // keys per KV block
constexpr int kHeadDim = 128;   // head dimension (fixed)
constexpr int kStages = 4;      // K/V ring depth
constexpr int kTileBytes = kBlockM * kHeadDim * 2;  // 32 KiB
constexpr int kHalfTileBytes = kTileBytes / 2;      // one TMA box: 64 cols x 128 rows
constexpr int kThreads = 384;    // 3 warpgroups
constexpr int kMmaWarp = 8;
constexpr int kLoadWarp = 9;     // warps 10-11 complete warpgroup 2 and idle
// Register split (setmaxnreg): launch 384 x 168 = 64512; softmax warpgroups
// 256 x 208 + warpgroup 2 128 x 88 = 64512.
constexpr uint32_t kLaunchRegs = 168;
constexpr uint32_t kSoftmaxRegs = 208;
constexpr uint32_t kControlRegs = 88;
static_assert(256 * kSoftmaxRegs + 128 * kControlRegs <= kThreads * kLaunchRegs, "register split exceeds the launch budget");
constexpr float kRescaleLog2 = 8.0f;  // lazy-rescale threshold (factor 256)

// Barrier slots.
constexpr int kBarQFull = 0;     // [2] Q tile landed                     (tx bytes)
constexpr int kBarQEmpty = 2;    // [2] Q buffer free                     (epilogue store issued)
constexpr int kBarSFull = 4;     // [2] S tile computed                   (tcgen05.commit)
constexpr int kBarPFull = 6;     // [2] P of keys 64-127 written          (128 threads)
constexpr int kBarOFinal = 8;    // [2] last PV of the item done          (tcgen05.commit)
constexpr int kBarOStaged = 10;  // [2] O tile staged in smem             (128 threads)
constexpr int kBarDrain = 12;    // MMA drain at exit                     (tcgen05.commit)
constexpr int kBarPHalf = 13;    // [2] P of keys 0-63 written, O corrected (128 threads)
constexpr int kBarTurn = 15;     // [2] softmax turn token of warpgroup t (128 threads)
constexpr int kBarKVFull = 17;   // [kStages]
constexpr int kBarKVEmpty = kBarKVFull + kStages;  // [kStages]
constexpr int kNumBars = kBarKVEmpty + kStages;

constexpr int kSmemQ = 0;
constexpr int kSmemKV = 2 * kTileBytes;
constexpr int kSmemBar = kSmemKV + kStages * kTileBytes;
constexpr int kSmemMisc = kSmemBar + kNumBars * 8;  // TMEM base (4 B), abort flag (4 B)
constexpr int kSmemUsed = kSmemMisc + 16;
constexpr int kSmemBytes = kSmemUsed + 1024;  // + slack for 1024-B alignment
static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
static_assert(kSmemBar % 8 == 0, "mbarrier alignment");

constexpr uint32_t kTmemCols = 512;

// tcgen05 instruction descriptors, kind::f16 (PTX ISA "Instruction
// descriptor"): bits 4-5 D format (1 = F32), 7-9 A format (0 = F16),
// 10-12 B format (0 = F16), 15 A major (0 = K), 16 B major (1 = MN),
// 17-22 N>>3, 24-28 M>>4.
constexpr uint32_t kIdescQK = (1u << 4) | (uint32_t(kBlockN >> 3) << 17) | (uint32_t(kBlockM >> 4) << 24);
constexpr uint32_t kIdescPV = (1u << 4) | (1u << 16) | (uint32_t(kHeadDim >> 3) << 17) | (uint32_t(kBlockM >> 4) << 24);

// Shared-memory matrix descriptors (PTX ISA "Matrix Descriptor"), 128-byte
// swizzle, sm_100 version bit.  Low word: start address >> 4 (bits 0-13),
// leading byte offset >> 4 (bits 16-29).  High word: stride byte offset >> 4
// (bits 0-13), version 1 (bit 14), layout SWIZZLE_128B = 2 (bits 29-31).
//  * K-major operand (Q, K): rows of 128 B, 8-row groups 1024 B apart (SBO);
//    the leading offset is unused for swizzled K-major layouts (set to 16 B).
//  * MN-major operand (V as the B matrix of P*V, head dim contiguous):
//    64-element column blocks kHalfTileBytes apart (LBO), 8-key groups
//    1024 B apart (SBO).
constexpr uint32_t kDescHi = uint32_t(1024 >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint32_t desc_lo_kmajor(uint32_t saddr) { return ((saddr & 0x3FFFFu) >> 4) | (1u << 16); }
__device__ __forceinline__ uint32_t desc_lo_mnmajor(uint32_t saddr) {
  return ((saddr & 0x3FFFFu) >> 4) | (uint32_t(kHalfTileBytes >> 4) << 16);
}

// exp2 on the FMA pipe for two lanes.  Cody-Waite split x = n + f with
// n = round(x) taken from the low mantissa bits of x + 1.5*2^23 and
// f = x - n in [-1/2, 1/2]; 2^f by the degree-3 minimax polynomial of
// fit_exp2_poly.py (relative error 7.5e-5, below FP16's half-ulp); n added to
// the exponent field as an integer.  x is clamped at -120 first so the
// exponent cannot wrap; 2^-120 is 0 in FP16 and negligible in the FP32 row
// sum, and masked keys (x = -inf) land there too.
constexpr int kPolyPairs = 2;  // of every 8 key pairs, these go to the polynomial
// The two softmax warpgroups share all four SMSPs; with kPingPong they take
// strict turns (tile 0, tile 1, tile 0, ...) so each runs at the full issue
// and MUFU rate while the tensor pipe works on the other tile.
constexpr bool kPingPong = false;
constexpr float kExp2C0 = 0.9999280571937561f;
constexpr float kExp2C1 = 0.6932609677314758f;
constexpr float kExp2C2 = 0.2426111251115799f;
constexpr float kExp2C3 = 0.0551716685295105f;

__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
  float a, b;
  f2_unpack(x2, a, b);
  const uint64_t xc = f2_pack(fmaxf(a, -120.f), fmaxf(b, -120.f));
  const uint64_t r = f2_add(xc, f2_pack(12582912.f, 12582912.f));     // round to integer
  const uint64_t nf = f2_add(r, f2_pack(-12582912.f, -12582912.f));   // n as a float
  const uint64_t f = f2_fma(nf, f2_pack(-1.f, -1.f), xc);             // x - n
  uint64_t q = f2_fma(f2_pack(kExp2C3, kExp2C3), f, f2_pack(kExp2C2, kExp2C2));
  q = f2_fma(q, f, f2_pack(kExp2C1, kExp2C1));
  q = f2_fma(q, f, f2_pack(kExp2C0, kExp2C0));
  float qa, qb, ra, rb;
  f2_unpack(q, qa, qb);
  f2_unpack(r, ra, rb);
  // r's bits are 0x4B400000 + n; times 2^23 only n << 23 survives (one mad).
  uint32_t ea, eb;
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(ea) : "r"(__float_as_uint(ra)), "r"(__float_as_uint(qa)));
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(eb) : "r"(__float_as_uint(rb)), "r"(__float_as_uint(qb)));
  return f2_pack(__uint_as_float(ea), __uint_as_float(eb));
}

struct FwdParams {
  CUtensorMap tm_q;  // (128, Nq, B*Hq)  fp16, box (64,128,1), 128-B swizzle
  CUtensorMap tm_k;  // (128, Nk, B*Hkv)
  CUtensorMap tm_v;  // (128, Nk, B*Hkv)
  CUtensorMap tm_o;  // (128, Nq, B*Hq)
  int32_t Hq, Hkv, group;   // group = Hq / Hkv
  int32_t nqb;              // ceil(Nq / 128)
  int32_t n_kv;             // ceil(Nk / 128)
  int32_t nk_tail;          // valid keys of the last KV block, 1..128
  int32_t unit_begin, unit_end;
  int32_t num_items;
  float scale_log2;         // scale * log2(e)
  uint32_t flags;
  uint64_t timeout_ns;
  uint32_t* ws;             // status header + trace records
};

constexpr uint32_t kFlagTrace = 1u;
constexpr uint32_t kFlagTestWithholdP = 2u;
constexpr uint32_t kFlagTimeline = 4u;

// Debug timeline (kFlagTimeline): CTA 0 stamps clock64() at fixed points of
// its first work item's first kTimelineBlocks key blocks.  Layout: u64
// [role][block][event] at byte kTimelineOffset of the workspace; roles
// 0/1 = softmax tile 0/1 (warp 4t, lane 0), 2 = MMA thread, 3 = TMA thread.
constexpr int kTimelineBlocks = 48;
constexpr uint32_t kTimelineOffset = 256u + 32u * 1024u;

struct Timeline {
  uint64_t* base;  // nullptr when not recording
  __device__ __forceinline__ void mark(int role, int j, int e) const {
    if (base != nullptr && j < kTimelineBlocks) base[(role * kTimelineBlocks + j) * 8 + e] = clock64();
  }
};

__device__ __forceinline__ Timeline make_timeline(const FwdParams& p, int it) {
  const bool on = (p.flags & kFlagTimeline) != 0 && blockIdx.x == 0 && it == 0;
  return Timeline{on ? reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(p.ws) + kTimelineOffset) : nullptr};
}

template <typename I>
__host__ __device__ __forceinline__ I ceil_div(I a, I b) {
  return (a + b - 1) / b;
}

// Work items of the unit range [ub, ue): pairs of consecutive units inside
// one head.  Closed form over (first partial head, full heads, last partial
// head) so that host and device agree without a table.
template <typename I>
__host__ __device__ inline I plan_count(I nqb, I ub, I ue) {
  if (ue <= ub) return 0;
  const I h0 = ub / nqb, h1 = (ue - 1) / nqb;
  const I hi0 = (ue < (h0 + 1) * nqb) ? ue : (h0 + 1) * nqb;
  I n = ceil_div<I>(hi0 - ub, 2);
  if (h1 > h0) n += (h1 - h0 - 1) * ceil_div<I>(nqb, 2) + ceil_div<I>(ue - h1 * nqb, 2);
  return n;
}

template <typename I>
__host__ __device__ inline void plan_decode(I nqb, I ub, I ue, I x, I& bh, I& qb, I& cnt) {
  const I h0 = ub / nqb, h1 = (ue - 1) / nqb;
  const I hi0 = (ue < (h0 + 1) * nqb) ? ue : (h0 + 1) * nqb;
  const I i0 = ceil_div<I>(hi0 - ub, 2);
  if (x < i0) {
    bh = h0;
    qb = ub - h0 * nqb + 2 * x;
    const I left = hi0 - h0 * nqb - qb;
    cnt = left < 2 ? left : 2;
    return;
  }
  x -= i0;
  const I per = ceil_div<I>(nqb, 2);
  const I mid = h1 - h0 - 1;
  if (x < mid * per) {
    bh = h0 + 1 + x / per;
    qb = 2 * (x % per);
    const I left = nqb - qb;
    cnt = left < 2 ? left : 2;
    return;
  }
  x -= mid * per;
  bh = h1;
  qb = 2 * x;
  const I left = ue - h1 * nqb - qb;
  cnt = left < 2 ? left : 2;
}

// Bounded mbarrier waits.  `site` identifies the wait in the status word:
// (warp << 8) | barrier slot.
struct Waiter {
  uint32_t abort_slot;  // shared u32, nonzero once any thread gave up
  uint64_t timeout_ns;
  uint32_t* ws;

  __device__ __forceinline__ void fail(uint32_t site) const {
    st_volatile_shared(abort_slot, 1u);
    if (atomicCAS(&ws[0], 0u, 1u /* B200FA_DEV_TIMEOUT */) == 0u) {
      ws[1] = site;
      ws[2] = blockIdx.x;
    }
    __threadfence();
  }

  __device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity, uint32_t site) const {
    if (mbar_test(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
#pragma unroll 1
      for (int i = 0; i < 16; ++i)
        if (mbar_test(bar, parity)) return true;
      if (ld_volatile_shared(abort_slot) != 0u) return false;
      if (global_timer_ns() - t0 > timeout_ns) {
        fail(site);
        return false;
      }
    }
  }

  // Exit-path wait for work this thread already issued (copies, MMAs); it
  // ignores the abort flag and gives up after `limit_ns`.
  __device__ __forceinline__ void drain(uint32_t bar, uint32_t parity, uint64_t limit_ns) const {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_test(bar, parity)) {
      if (global_timer_ns() - t0 > limit_ns) return;
    }
  }
};

struct Smem {
  uint32_t base;  // shared-window address of the aligned base
  __device__ __forceinline__ uint32_t bar(int i) const { return base + kSmemBar + 8 * i; }
  __device__ __forceinline__ uint32_t q(int t) const { return base + kSmemQ + t * kTileBytes; }
  __device__ __forceinline__ uint32_t kv(uint32_t s) const { return base + kSmemKV + s * kTileBytes; }
  __device__ __forceinline__ uint32_t tmem_slot() const { return base + kSmemMisc; }
  __device__ __forceinline__ uint32_t abort_slot() const { return base + kSmemMisc + 4; }

};

// ------------------------------------------------------------------ roles
// S = Q K^T over the full head dim (8 K-major steps, overwrite).
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_smem, uint32_t k_smem) {
  mma_ss_k128(d_tmem, desc_lo_kmajor(q_smem), desc_lo_kmajor(k_smem), kDescHi, kIdescQK, 0u);
}

// O (+)= P V over keys [64*half, 64*half + 64): A = P's TMEM columns
// [64*half, 64*half + 32) (FP16 pairs; each key half's P sits at the start of
// that half's own S columns), B = V rows of those keys.
template <int half>
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_smem, bool accumulate) {
  mma_ts_k64(d_tmem, p_tmem + 64 * half, desc_lo_mnmajor(v_smem) + 512 * half, kDescHi, kIdescPV,
             (half > 0 || accumulate) ? 1u : 0u);
}

__device__ void mma_role(const FwdParams& p, const Smem& sm, uint32_t tmem_base, const Waiter& w) {
  const uint32_t tS0 = tmem_base, tS1 = tmem_base + 128;
  const uint32_t tO0 = tmem_base + 256, tO1 = tmem_base + 384;
  const uint32_t site = uint32_t(kMmaWarp) << 8;
  const int n = p.n_kv;
  uint32_t kv_it = 0;
  uint32_t p_phase = 0;  // bit t: phase of P-full[t]
  bool ok = true;
  for (int item = blockIdx.x, it = 0; ok && item < p.num_items; item += gridDim.x, ++it) {
    const Timeline tl = make_timeline(p, it);
    const uint32_t ip = uint32_t(it) & 1u;
    uint32_t sk = kv_it % kStages;
    if (!w.wait(sm.bar(kBarQFull + 0), ip, site | (kBarQFull + 0))) break;
    if (!w.wait(sm.bar(kBarKVFull + sk), (kv_it / kStages) & 1u, site | (kBarKVFull + sk))) break;
    tc_fence_after();
    issue_qk(tS0, sm.q(0), sm.kv(sk));
    mma_commit(sm.bar(kBarSFull + 0));
    if (!w.wait(sm.bar(kBarQFull + 1), ip, site | (kBarQFull + 1))) break;
    tc_fence_after();
    issue_qk(tS1, sm.q(1), sm.kv(sk));
    mma_commit(sm.bar(kBarSFull + 1));
    mma_commit(sm.bar(kBarKVEmpty + sk));
    ++kv_it;
    for (int j = 0; j < n; ++j) {
      tl.mark(2, j, 0);
      const uint32_t sv = kv_it % kStages;
      const uint32_t vph = (kv_it / kStages) & 1u;
      ++kv_it;
      if (!w.wait(sm.bar(kBarKVFull + sv), vph, site | (kBarKVFull + sv))) { ok = false; break; }
      tl.mark(2, j, 1);
      if (!w.wait(sm.bar(kBarPHalf + 0), p_phase & 1u, site | (kBarPHalf + 0))) { ok = false; break; }
      tl.mark(2, j, 2);
      tc_fence_after();
      issue_pv<0>(tO0, tS0, sm.kv(sv), j > 0);
      if (!w.wait(sm.bar(kBarPFull + 0), p_phase & 1u, site | (kBarPFull + 0))) { ok = false; break; }
      tl.mark(2, j, 3);
      p_phase ^= 1u;
      tc_fence_after();
      issue_pv<1>(tO0, tS0, sm.kv(sv), true);
      if (j == n - 1) mma_commit(sm.bar(kBarOFinal + 0));
      const bool more = j + 1 < n;
      uint32_t sk2 = 0;
      if (more) {
        sk2 = kv_it % kStages;
        if (!w.wait(sm.bar(kBarKVFull + sk2), (kv_it / kStages) & 1u, site | (kBarKVFull + sk2))) {
          ok = false;
          break;
        }
        tl.mark(2, j, 4);
        tc_fence_after();
        issue_qk(tS0, sm.q(0), sm.kv(sk2));
        mma_commit(sm.bar(kBarSFull + 0));
      }
      if (!w.wait(sm.bar(kBarPHalf + 1), (p_phase >> 1) & 1u, site | (kBarPHalf + 1))) { ok = false; break; }
      tl.mark(2, j, 5);
      tc_fence_after();
      issue_pv<0>(tO1, tS1, sm.kv(sv), j > 0);
      if (!w.wait(sm.bar(kBarPFull + 1), (p_phase >> 1) & 1u, site | (kBarPFull + 1))) { ok = false; break; }
      tl.mark(2, j, 6);
      p_phase ^= 2u;
      tc_fence_after();
      issue_pv<1>(tO1, tS1, sm.kv(sv), true);
      mma_commit(sm.bar(kBarKVEmpty + sv));
      if (j == n - 1) mma_commit(sm.bar(kBarOFinal + 1));
      if (more) {
        issue_qk(tS1, sm.q(1), sm.kv(sk2));
        mma_commit(sm.bar(kBarSFull + 1));
        mma_commit(sm.bar(kBarKVEmpty + sk2));
        tl.mark(2, j, 7);
        ++kv_it;
      }
    }
  }
  // All MMAs this thread issued must be complete before TMEM is freed.
  mma_commit(sm.bar(kBarDrain));
  w.drain(sm.bar(kBarDrain), 0u, 100000000ull);
}

__device__ void load_role(const FwdParams& p, const Smem& sm, const Waiter& w) {
  const uint32_t site = uint32_t(kLoadWarp) << 8;
  const int n = p.n_kv;
  uint32_t kv_it = 0;
  uint32_t issued = 0;       // bit s: stage s has ever been loaded
  uint32_t last_par = 0;     // bit s: parity of stage s's last load
  uint32_t q_issued = 0, q_par = 0;
  bool ok = true;
  for (int item = blockIdx.x, it = 0; ok && item < p.num_items; item += gridDim.x, ++it) {
    int bh, qb, cnt;
    plan_decode<int>(p.nqb, p.unit_begin, p.unit_end, item, bh, qb, cnt);
    const int b = bh / p.Hq;
    const int kvh = b * p.Hkv + (bh - b * p.Hq) / p.group;
    const int row0 = qb * kBlockM;
    const int row1 = cnt == 2 ? row0 + kBlockM : row0;
    const uint32_t ip = uint32_t(it) & 1u;
    const Timeline tl = make_timeline(p, it);
    if (!w.wait(sm.bar(kBarQEmpty + 0), ip ^ 1u, site | (kBarQEmpty + 0))) break;
    mbar_arrive_expect_tx(sm.bar(kBarQFull + 0), kTileBytes);
    tma_load_3d(sm.q(0), &p.tm_q, sm.bar(kBarQFull + 0), 0, row0, bh);
    tma_load_3d(sm.q(0) + kHalfTileBytes, &p.tm_q, sm.bar(kBarQFull + 0), 64, row0, bh);
    q_issued |= 1u;
    q_par = (q_par & ~1u) | ip;
    for (int j = 0; j < n; ++j) {
#pragma unroll
      for (int which = 0; which < 2; ++which) {  // 0: K_j, 1: V_j
        const uint32_t s = kv_it % kStages;
        const uint32_t ph = (kv_it / kStages) & 1u;
        ++kv_it;
        tl.mark(3, j, 2 * which);
        if (!w.wait(sm.bar(kBarKVEmpty + s), ph ^ 1u, site | (kBarKVEmpty + s))) { ok = false; break; }
        tl.mark(3, j, 2 * which + 1);
        const CUtensorMap* map = which == 0 ? &p.tm_k : &p.tm_v;
        mbar_arrive_expect_tx(sm.bar(kBarKVFull + s), kTileBytes);
        tma_load_3d(sm.kv(s), map, sm.bar(kBarKVFull + s), 0, j * kBlockN, kvh);
        tma_load_3d(sm.kv(s) + kHalfTileBytes, map, sm.bar(kBarKVFull + s), 64, j * kBlockN, kvh);
        issued |= 1u << s;
        last_par = (last_par & ~(1u << s)) | (ph << s);
        if (which == 0 && j == 0) {
          if (!w.wait(sm.bar(kBarQEmpty + 1), ip ^ 1u, site | (kBarQEmpty + 1))) { ok = false; break; }
          mbar_arrive_expect_tx(sm.bar(kBarQFull + 1), kTileBytes);
          tma_load_3d(sm.q(1), &p.tm_q, sm.bar(kBarQFull + 1), 0, row1, bh);
          tma_load_3d(sm.q(1) + kHalfTileBytes, &p.tm_q, sm.bar(kBarQFull + 1), 64, row1, bh);
          q_issued |= 2u;
          q_par = (q_par & ~2u) | (ip << 1);
        }
      }
      if (!ok) break;
    }
  }
  // Copies still in flight must land before the CTA exits (only possible on
  // the abort path; on the normal path the MMA thread consumed every stage).
  if (!ok || ld_volatile_shared(sm.abort_slot()) != 0u) {
    for (int s = 0; s < kStages; ++s)
      if (issued & (1u << s)) w.drain(sm.bar(kBarKVFull + s), (last_par >> s) & 1u, 50000000ull);
    for (int t = 0; t < 2; ++t)
      if (q_issued & (1u << t)) w.drain(sm.bar(kBarQFull + t), (q_par >> t) & 1u, 50000000ull);
  }
}

// Exponentials of 64 keys (32 pairs) of one row: x = s * scale*log2(e) - m
// with packed FP32 FMAs; of every 8 pairs the last kPoly go through the
// FMA-pipe polynomial (exp2_poly2) and the rest through MUFU (FP32 ex2, or
// FP16x2 ex2 in the FP16 variant).  Writes 32 packed FP16 pairs of P and adds
// to the running row-sum accumulators.
template <int kVariant, int kPoly>
__device__ __forceinline__ void exp_keys64(const uint32_t* r, uint64_t sl2x2, uint64_t nmx2, uint32_t* pk,
                                           uint64_t& acc0, uint64_t& acc1, float& hsum) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t hacc = 0u;
#pragma unroll
    for (int pp = 0; pp < 8; ++pp) {
      const int i = g * 8 + pp;  // key pair index within the 64 keys
      const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), sl2x2, nmx2);
      if (pp >= 8 - kPoly) {
        const uint64_t p2 = exp2_poly2(x2);
        if (pp & 1) acc1 = f2_add(acc1, p2); else acc0 = f2_add(acc0, p2);
        float a, b;
        f2_unpack(p2, a, b);
        pk[i] = pack_h2(a, b);
      } else if constexpr (kVariant == 1) {
        float a, b;
        f2_unpack(x2, a, b);
        const float ea = ex2_approx(a), eb = ex2_approx(b);
        const uint64_t p2 = f2_pack(ea, eb);
        if (pp & 1) acc1 = f2_add(acc1, p2); else acc0 = f2_add(acc0, p2);
        pk[i] = pack_h2(ea, eb);
      } else {
        float a, b;
        f2_unpack(x2, a, b);
        const uint32_t e2 = ex2_approx_h2(pack_h2(a, b));
        pk[i] = e2;
        hacc = (pp == 0) ? e2 : hadd2(hacc, e2);
      }
    }
    if constexpr (kVariant == 0) {
      if (kPoly < 8) hsum += h2_sum_f32(hacc);
    }
  }
}

// Keys at or beyond `valid` (the last block's key count) get score -inf.
__device__ __forceinline__ void mask_keys(uint32_t* r, int first_key, int valid) {
#pragma unroll
  for (int i = 0; i < 64; ++i)
    if (first_key + i >= valid) r[i] = __float_as_uint(-INFINITY);
}

// Row maximum of 64 scores: 3-input max, four independent chains.
__device__ __forceinline__ float row_max64(const uint32_t* r) {
  float mc0 = -INFINITY, mc1 = -INFINITY, mc2 = -INFINITY, mc3 = -INFINITY;
#pragma unroll
  for (int i = 0; i < 64; i += 8) {
    mc0 = max3(mc0, __uint_as_float(r[i + 0]), __uint_as_float(r[i + 1]));
    mc1 = max3(mc1, __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
    mc2 = max3(mc2, __uint_as_float(r[i + 4]), __uint_as_float(r[i + 5]));
    mc3 = max3(mc3, __uint_as_float(r[i + 6]), __uint_as_float(r[i + 7]));
  }
  return fmaxf(fmaxf(mc0, mc1), fmaxf(mc2, mc3));
}

// Softmax of one query tile per warpgroup (warps 0-3: tile 0, 4-7: tile 1),
// one thread per query row (its TMEM lane), all 128 keys of a block.
//
// After a tile's first block the exponentials of keys 0-63 are computed
// speculatively against the current reference maximum while the block's row
// maximum is reduced; they are redone only if that maximum exceeds the
// reference by more than 2^kRescaleLog2 (rare once it has settled).  P goes to
// the MMA warp in two halves: keys 0-63 into TMEM columns 0-31 of the tile's
// S region, keys 64-127 into columns 64-95.
template <int kVariant>  // 0 = FP16 softmax, 1 = FP32 softmax
__device__ void softmax_role(const FwdParams& p, const Smem& sm, uint32_t tmem_base, const Waiter& w,
                             uint32_t warp, uint32_t lane) {
  const int t = int(warp >> 2);   // tile = warpgroup
  const int wq = int(warp & 3);   // TMEM lane quarter of this warp
  const int row = wq * 32 + int(lane);
  const uint32_t lane_off = uint32_t(wq * 32) << 16;
  const uint32_t tS = tmem_base + lane_off + uint32_t(t) * 128;
  const uint32_t tO = tmem_base + lane_off + 256 + uint32_t(t) * 128;
  const uint32_t sQ = sm.q(t);
  const uint32_t site = warp << 8;
  const float sl2 = p.scale_log2;
  const uint64_t sl2x2 = f2_pack(sl2, sl2);
  const int n = p.n_kv;
  const bool withhold = (p.flags & kFlagTestWithholdP) != 0 && t == 1;
  uint32_t s_phase = 0;
  uint32_t turns = 0;  // ping-pong turns taken
  bool ok = true;

  for (int item = blockIdx.x, it = 0; ok && item < p.num_items; item += gridDim.x, ++it) {
    float m_ref = -INFINITY;  // reference maximum, log2 domain
    float l = 0.f;
    const Timeline tl = (wq == 0 && lane == 0) ? make_timeline(p, it) : Timeline{nullptr};
    for (int j = 0; j < n; ++j) {
      if (!w.wait(sm.bar(kBarSFull + t), s_phase, site | (kBarSFull + t))) { ok = false; break; }
      tl.mark(t, j, 0);
      s_phase ^= 1u;
      if (kPingPong) {  // warpgroup 0's first turn is free (parity trick)
        if (!w.wait(sm.bar(kBarTurn + t), (turns & 1u) ^ (t == 0 ? 1u : 0u), site | (kBarTurn + t))) { ok = false; break; }
        ++turns;
      }
      tc_fence_after();
      // Keys 0-63: load, exponentiate speculatively against the current
      // reference (after the first block), and reduce their maximum.
      const bool tail = (j == n - 1 && p.nk_tail < kBlockN);
      uint32_t pk[64];
      uint64_t acc0 = 0ull, acc1 = 0ull;  // packed FP32 partial row sums
      float hsum = 0.f;                   // FP16 variant: sums of FP16 group sums
      float mx;
      {
        uint32_t r[64];
        tmem_ld32(tS + 0, r + 0);
        tmem_ld32(tS + 32, r + 32);
        tmem_wait_ld();
        tl.mark(t, j, 1);
        if (tail) mask_keys(r, 0, p.nk_tail);
        if (j > 0) exp_keys64<kVariant, kPolyPairs>(r, sl2x2, f2_pack(-m_ref, -m_ref), pk, acc0, acc1, hsum);
        mx = row_max64(r);
      }
      // Keys 64-127: load and reduce (their exponentials follow the check).
      uint32_t r1[64];
      tmem_ld32(tS + 64, r1 + 0);
      tmem_ld32(tS + 96, r1 + 32);
      tmem_wait_ld();
      if (tail) mask_keys(r1, 64, p.nk_tail);
      const float m_blk = fmaxf(mx, row_max64(r1)) * sl2;
      float alpha = 1.f;
      bool moved = false;
      if (m_blk > m_ref + kRescaleLog2) {
        alpha = ex2_approx(m_ref - m_blk);  // 0 on the first block
        m_ref = m_blk;
        moved = true;
      }
      l *= alpha;
      tl.mark(t, j, 2);
      // Lazy correction of the running output before any of this block's P
      // is handed over.  PV_t(j-1) is complete: the commit that signalled
      // S_t(j) covers it.  The P stores' wait below also covers these stores.
      if (j > 0 && __any_sync(0xffffffffu, moved)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + 32 * c, o);
        }
      }
      if (__any_sync(0xffffffffu, moved)) {
        // First block, or the reference moved: recompute keys 0-63 from S,
        // which is still in TMEM (P has not been written yet).
        uint32_t r[64];
        tmem_ld32(tS + 0, r + 0);
        tmem_ld32(tS + 32, r + 32);
        tmem_wait_ld();
        if (tail) mask_keys(r, 0, p.nk_tail);
        if (moved) {
          acc0 = 0ull;
          acc1 = 0ull;
          hsum = 0.f;
          exp_keys64<kVariant, kPolyPairs>(r, sl2x2, f2_pack(-m_ref, -m_ref), pk, acc0, acc1, hsum);
        }
      }
      tmem_st32(tS, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(sm.bar(kBarPHalf + t));
      tl.mark(t, j, 3);
      exp_keys64<kVariant, kPolyPairs>(r1, sl2x2, f2_pack(-m_ref, -m_ref), pk + 32, acc0, acc1, hsum);
      tmem_st32(tS + 64, pk + 32);
      tmem_wait_st();
      tc_fence_before();
      if (!(withhold && it == 0 && j == 0)) mbar_arrive(sm.bar(kBarPFull + t));
      if (kPingPong) mbar_arrive(sm.bar(kBarTurn + (1 - t)));
      tl.mark(t, j, 4);
      float a0, b0, a1, b1;
      f2_unpack(acc0, a0, b0);
      f2_unpack(acc1, a1, b1);
      l += ((a0 + b0) + (a1 + b1)) + hsum;
    }
    if (!ok) break;

    // ---- epilogue: O / l -> FP16 -> swizzled smem (this tile's Q buffer) -> TMA store
    if (!w.wait(sm.bar(kBarOFinal + t), uint32_t(it) & 1u, site | (kBarOFinal + t))) { ok = false; break; }
    tc_fence_after();
    const float inv_l = 1.f / l;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t o[32];
      tmem_ld32(tO + 32 * c, o);
      tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t h0 = pack_h2(__uint_as_float(o[8 * u + 0]) * inv_l, __uint_as_float(o[8 * u + 1]) * inv_l);
        const uint32_t h1 = pack_h2(__uint_as_float(o[8 * u + 2]) * inv_l, __uint_as_float(o[8 * u + 3]) * inv_l);
        const uint32_t h2 = pack_h2(__uint_as_float(o[8 * u + 4]) * inv_l, __uint_as_float(o[8 * u + 5]) * inv_l);
        const uint32_t h3 = pack_h2(__uint_as_float(o[8 * u + 6]) * inv_l, __uint_as_float(o[8 * u + 7]) * inv_l);
        const int gu = c * 4 + u;  // 16-byte unit of the 256-byte output row
        const uint32_t addr = sQ + uint32_t(gu >> 3) * kHalfTileBytes + uint32_t(row) * 128 +
                              (uint32_t((gu & 7) ^ (row & 7)) << 4);
        st_shared_v4(addr, h0, h1, h2, h3);
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(sm.bar(kBarOStaged + t));
    if (wq == 0 && lane == 0) {
      int bh, qb, cnt;
      plan_decode<int>(p.nqb, p.unit_begin, p.unit_end, item, bh, qb, cnt);
      if (!w.wait(sm.bar(kBarOStaged + t), uint32_t(it) & 1u, site | (kBarOStaged + t))) {
        ok = false;
      } else {
        if (t == 0 || cnt == 2) {
          const int orow = qb * kBlockM + t * kBlockM;
          tma_store_3d(&p.tm_o, sQ, 0, orow, bh);
          tma_store_3d(&p.tm_o, sQ + kHalfTileBytes, 64, orow, bh);
          bulk_commit_group();
          bulk_wait_group_read0();
        }
        mbar_arrive(sm.bar(kBarQEmpty + t));
      }
    }
  }
  if (wq == 0 && lane == 0) bulk_wait_group0();
}

template <int kVariant>
__device__ __forceinline__ void attention_fwd_body(const FwdParams& p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  Smem sm{(raw + 1023u) & ~1023u};
  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t t_start = global_timer_ns();

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(sm.bar(kBarQFull + t), 1);
      mbar_init(sm.bar(kBarQEmpty + t), 1);
      mbar_init(sm.bar(kBarSFull + t), 1);
      mbar_init(sm.bar(kBarPFull + t), 128);
      mbar_init(sm.bar(kBarPHalf + t), 128);
      mbar_init(sm.bar(kBarOFinal + t), 1);
      mbar_init(sm.bar(kBarOStaged + t), 128);
      mbar_init(sm.bar(kBarTurn + t), 128);
    }
    mbar_init(sm.bar(kBarDrain), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(sm.bar(kBarKVFull + s), 1);
      mbar_init(sm.bar(kBarKVEmpty + s), 1);
    }
    st_volatile_shared(sm.abort_slot(), 0u);
    fence_mbarrier_init();
  }
  if (warp == kLoadWarp && lane == 0) {
    tma_prefetch_map(&p.tm_q);
    tma_prefetch_map(&p.tm_k);
    tma_prefetch_map(&p.tm_v);
    tma_prefetch_map(&p.tm_o);
  }
  if (warp == 0) {
    tmem_alloc(sm.tmem_slot(), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ld_volatile_shared(sm.tmem_slot());
  const Waiter w{sm.abort_slot(), p.timeout_ns, p.ws};

  if (warp < 8) {
    regs_increase<kSoftmaxRegs>();
    softmax_role<kVariant>(p, sm, tmem_base, w, warp, lane);
  } else {
    regs_decrease<kControlRegs>();
    if (warp == kMmaWarp) {
      if (lane == 0) mma_role(p, sm, tmem_base, w);
    } else if (warp == kLoadWarp) {
      if (lane == 0) load_role(p, sm, w);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if ((p.flags & kFlagTrace) && threadIdx.x == kLoadWarp * 32 && blockIdx.x < 1024) {
    uint32_t* rec = p.ws + (256 + 32 * blockIdx.x) / 4;
    int items = 0;
    for (int item = blockIdx.x; item < p.num_items; item += gridDim.x) ++items;
    const uint64_t t_end = global_timer_ns();
    rec[0] = sm_id();
    rec[1] = uint32_t(items);
    rec[2] = uint32_t(t_start);
    rec[3] = uint32_t(t_start >> 32);
    rec[4] = uint32_t(t_end);
    rec[5] = uint32_t(t_end >> 32);
    rec[6] = 0u;
    rec[7] = 0u;
  }
}

}  // namespace b200fa
