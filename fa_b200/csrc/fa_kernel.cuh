// fa_kernel.cuh -- the sm_100a warp-specialised flash-attention forward.
//
// Operator (reference semantics: backends/npu_fa/backend.py:36-49, FP32
// formula backends/expert_v2/impl_tl.py:701-717):
//   O[b,h] = softmax(Q[b,h] K[b,kv]^T * scale) V[b,kv],  kv = b*Hkv + h/(Hq/Hkv)
// (GQA head map of panel_kernel.h:274), non-causal, D = 128, FP16 in/out.
//
// Work decomposition.  A work unit is one 128-row query block of one (b, hq),
// linearised ((b*Hq)+hq)*ceil(Nq/128)+qb (cce_task.h:28-35 order).  A work
// item is two consecutive units of the same head, one per CTA of a pair,
// sharing every K/V block.  Items are dealt round-robin to a persistent grid
// of CTA pairs (clusters of two CTAs on the two SMs of a TPC), one pair per
// TPC.
//
// The pair.  Both tensor-core products run as pair MMAs (tcgen05
// cta_group::2, M = 256) issued by rank 0: each CTA holds its unit's 128
// query rows, and the B operand is split between the two shared memories --
// rank r holds keys [64r, 64r+64) of every 128-key K block (S = Q K^T, one
// N = 128 product per block) and head-dim columns [64r, 64r+64) of every V
// block (O = P V).  Per SM and K=16 step the S product reads 4 KiB of Q and
// 2 KiB of K from shared memory (48 cycles at 128 B/clk against 64 of tensor
// work), and each SM loads only half of every K/V block.
//
// CTA roles (384 threads = 3 warpgroups), the same in both CTAs:
//   warps 0-3   softmax group 0: the item's even key blocks (TMEM lanes = rows)
//   warps 4-7   softmax group 1: the odd key blocks
//   warp  8     rank 0: the S issuer (one thread): every S = Q K^T product
//   warp  9     TMA producer (one thread): this CTA's Q tiles and K/V halves
//   warp  10    rank 0: the PV issuer (one thread): every O += P V product
//   warp  11    rank 1: forwards its TMA completions to rank 0's barriers
//
// Schedule.  The CTA counts its key blocks over all its items; block g has
// its scores in S buffer g % 2 and its P in P buffer g % 2 (both in tensor
// memory).  The S issuer writes S of block g once the softmax has read the
// scores of block g - 2 from that buffer ("S free"), so scores run up to two
// blocks ahead of the softmax; the PV issuer runs O += P V for block g once
// its P is written ("P full") and then reports the P buffer free and O up
// to date ("PV done").  Each kind of product has its own issuing thread: a
// single thread whose stream alternates S and PV products feeds the tensor
// pipe far below its rate (measured on B200: ~100 cycles per N = 128 pair
// product instead of ~65); two threads with one kind each keep it busy.
// The two softmax groups take alternate blocks, each with two block periods
// for its block; both run at once on every SM sub-partition, so each hides
// the other's latencies.  K and V have separate rings: a K stage is free
// once S of its block completed, a V stage once PV did.  Rank 1's TMA
// completions reach rank 0 through its warp 11, which waits for each local
// stage and arrives on rank 0's barrier: no copy ever signals the other CTA.
//
// Tensor memory (same columns in both CTAs):
//   O   [0, 128)             FP32 output accumulator
//   P_b [128 + 64b, +64)     FP16 P of a block (pairs), b = 0, 1
//   S_b [256 + 128b, +128)   FP32 scores of a 128-key block (key c in column c)
//
// Shared memory (1024-B aligned, 128-byte swizzle as the TMA writes it):
//   two Q tiles (32 KiB each: two 64-column halves of 128 rows; item i uses
//   tile i % 2, so the next item's Q lands while this one runs, and the tile
//   stages the item's FP16 output for the TMA store), a K ring and a V ring
//   of kRing stages each (16 KiB: this CTA's 64 keys of a block, as two
//   64-column boxes, / this CTA's 64 head-dim columns of the block's 128
//   keys), the softmax groups' exchange area, mbarriers.
//
// Online softmax (per query row, one thread per row in each group): the
// reference maximum m (log2 domain) moves only when a block's maximum
// exceeds it by more than kRescaleLog2 (lazy rescaling), so P <=
// 2^kRescaleLog2 and O/l is exact at the end whatever the reference.  The
// reference after block g is passed to the other group through shared memory
// ("ref g"); the group that moves it rescales the row's O in TMEM (after
// PV of block g-1 completed) before its P is handed over.  Each group keeps
// its own partial row sum, relative to the reference of its last block; the
// two are brought to the final reference and added at the end of the item.
//
// Every wait is bounded (global timer); on expiry the kernel records
// B200FA_DEV_TIMEOUT in the workspace, raises the abort flag of both CTAs,
// every role leaves its loop, in-flight copies and MMAs are drained with a
// second bound, TMEM is freed and the kernel returns.  The checking build
// (B200FA_DEBUG) also verifies coordinates, indices and layout before use
// and the roles' block counts at exit (B200FA_DEV_BOUNDS / _PHASE).
#pragma once
#include <cstdint>
#include <cuda.h>
#include "ptx.cuh"

// B200FA_CAUSAL = 1: this translation unit's kernels apply the causal mask
// (query row i attends keys 0..i).  The causal kernels are compiled in their
// own translation unit (b200fa_causal.cu), so that the product kernels are
// compiled from exactly the non-causal source: the pipeline's timing is
// sensitive to the instruction schedule, and folding the option into one
// source moved the product kernels by 2 % (A/B on one box).
#ifndef B200FA_CAUSAL
#define B200FA_CAUSAL 0
#endif

namespace b200fa {

constexpr int kBlockM = 128;    // query rows per unit (per CTA)
constexpr int kBlockN = 128;    // keys per KV block
constexpr int kHeadDim = 128;   // head dimension (fixed)
constexpr int kPairKeys = kBlockN / 2;    // K rows of a block held by each CTA
constexpr int kPairDims = kHeadDim / 2;   // V head-dim columns held by each CTA
constexpr int kItemUnits = 2;   // query units per work item (one per CTA)
constexpr int kRing = 5;        // entries of the K ring and of the V ring (one stage each)
constexpr int kQTileBytes = kBlockM * kHeadDim * 2;   // 32 KiB
constexpr int kQHalfBytes = kQTileBytes / 2;          // TMA box: 64 cols x 128 rows
constexpr int kKBoxRows = kPairKeys;                  // K rows of a block held by each CTA
constexpr int kKBoxBytes = kKBoxRows * 128;           // TMA box: 64 cols x 64 rows
constexpr int kStageBytes = 2 * kKBoxBytes;           // 16 KiB
static_assert(kBlockN * kPairDims * 2 == kStageBytes, "K and V stages must have the same size");
constexpr int kThreads = 384;      // 3 warpgroups
constexpr int kSIssuerWarp = 8;    // rank 0: issues every S product
constexpr int kLoadWarp = 9;
constexpr int kPVIssuerWarp = 10;  // rank 0: issues every PV product
constexpr int kForwardWarp = 11;   // rank 1
// Register split (setmaxnreg): launch 384 x 168 = 64512; softmax warpgroups
// 256 x 208 + warpgroup 2 128 x 88 = 64512.  ptxas holds each region to its
// share (both build flavours compile spill-free at this split).
#ifndef B200FA_SOFTMAX_REGS
#define B200FA_SOFTMAX_REGS 208
#endif
constexpr uint32_t kLaunchRegs = 168;
constexpr uint32_t kSoftmaxRegs = B200FA_SOFTMAX_REGS;
constexpr uint32_t kControlRegs = (kThreads * kLaunchRegs - 256 * kSoftmaxRegs) / 128 / 8 * 8;
static_assert(256 * kSoftmaxRegs + 128 * kControlRegs <= kThreads * kLaunchRegs, "register split exceeds the launch budget");
constexpr float kRescaleLog2 = 8.0f;  // lazy-rescale threshold (factor 256)

// Tensor memory columns.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 0;       // O, 128 columns
constexpr uint32_t kTmemP = 128;     // + 64 b: P buffer b (FP16 pairs, 64 columns)
constexpr uint32_t kTmemS = 256;     // + 128 b: S buffer b (FP32, 128 columns)
static_assert(kTmemS + 2 * 128 <= kTmemCols, "TMEM budget");

// Barrier slots.  "rank 0" barriers are only waited on in rank 0.
constexpr int kBarQFull = 0;     // [2] Q tile landed (rank 0: own TMA + rank 1's forward; rank 1: own TMA)
constexpr int kBarQEmpty = 2;    // [2] Q tile free (the epilogue's store read it)                local
constexpr int kBarSFull = 4;     // [2] S buffer b computed                    (S issuer commit to both CTAs)
constexpr int kBarSFree = 6;     // [2] rank 0: S buffer b read by one group's 4 warps in each CTA
constexpr int kBarPFull = 8;     // [2] rank 0: P buffer b written by one group's 4 warps in each CTA
constexpr int kBarPVDone = 10;   // [2] PV of P buffer b done; O holds every block so far (PV issuer commit)
constexpr int kBarRef = 12;      // [2] reference maximum of block g published (g % 2; 4 warps)  local
constexpr int kBarXchg = 14;     // [1] epilogue row-sum exchange (8 warps)                        local
constexpr int kBarOStaged = 15;  // [1] O tile staged in smem (8 warps)                            local
constexpr int kBarDrain = 16;    // [2] rank 0: MMA drain of the S / PV issuer at exit
constexpr int kBarKFull = 18;    // [kRing] K stage landed (rank 0: own TMA + rank 1's forward)
constexpr int kBarKEmpty = kBarKFull + kRing;   // [kRing] S of its block done (S issuer commit to both CTAs)
constexpr int kBarVFull = kBarKEmpty + kRing;   // [kRing] V stage landed (rank 0: own TMA + rank 1's forward)
constexpr int kBarVEmpty = kBarVFull + kRing;   // [kRing] PV of its block done (PV issuer commit to both CTAs)
constexpr int kNumBars = kBarVEmpty + kRing;
constexpr uint32_t kGroupWarps = 8;  // one group's warps in the pair (arrivals on "S free" / "P full")

constexpr int kSmemQ = 0;
constexpr int kSmemK = 2 * kQTileBytes;
constexpr int kSmemV = kSmemK + kRing * kStageBytes;
constexpr int kSmemBar = kSmemV + kRing * kStageBytes;
constexpr int kSmemXchg = kSmemBar + kNumBars * 8;        // float [2][128] reference / row-sum exchange
constexpr int kSmemMisc = kSmemXchg + 2 * kBlockM * 4;    // TMEM base, abort flag, 6 block counters
constexpr int kSmemUsed = kSmemMisc + 8 + 4 * 6 + 8;  // + start time (trace)
constexpr int kSmemBytes = kSmemUsed + 1024;  // + slack for 1024-B alignment
static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
static_assert(kSmemBar % 8 == 0, "mbarrier alignment");
static_assert(kKBoxBytes % 1024 == 0 && kStageBytes % 1024 == 0, "128-byte swizzle atoms must stay 1024-B aligned");

// tcgen05 instruction descriptors, kind::f16 (PTX ISA "Instruction
// descriptor"): bits 4-5 D format (1 = F32), 7-9 A format (0 = F16),
// 10-12 B format (0 = F16), 15 A major (0 = K), 16 B major (1 = MN),
// 17-22 N>>3, 24-28 M>>4.  M = 256: the pair's rows; N = 128 for both
// products (S: the block's keys, 64 per CTA; PV: the head dims, 64 per CTA).
constexpr uint32_t kIdescQK = (1u << 4) | (uint32_t(kBlockN >> 3) << 17) | (uint32_t(256 >> 4) << 24);
constexpr uint32_t kIdescPV = (1u << 4) | (1u << 16) | (uint32_t(kHeadDim >> 3) << 17) | (uint32_t(256 >> 4) << 24);
static_assert(kBlockN % 16 == 0 && kBlockN <= 256, "M=256 needs N a multiple of 16");

// Shared-memory matrix descriptors (PTX ISA "Matrix Descriptor"), 128-byte
// swizzle, sm_100 version bit.  Low word: start address >> 4 (bits 0-13),
// leading byte offset >> 4 (bits 16-29).  High word: stride byte offset >> 4
// (bits 0-13), version 1 (bit 14), layout SWIZZLE_128B = 2 (bits 29-31).
// Rows of 128 B, 8-row groups 1024 B apart (SBO) for Q, K (K-major) and V
// (MN-major: rows are keys, 64 head-dim columns per row).  The leading
// offset is unused: swizzled K-major layouts ignore it and each CTA's V
// half is a single 64-column block; it is set to 16 B.  Offsets added to a
// descriptor's start address never carry out of bits 0-13: shared addresses
// are below 256 KiB.
constexpr uint32_t kDescHi = uint32_t(1024 >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
  return (uint64_t(kDescHi) << 32) | uint64_t(((saddr & 0x3FFFFu) >> 4) | (1u << 16));
}

// exp2 on the FMA pipe for two lanes.  Cody-Waite split x = n + f with
// n = round(x) taken from the low mantissa bits of x + 1.5*2^23 and
// f = x - n in [-1/2, 1/2]; 2^f by the degree-3 minimax polynomial of
// fit_exp2_poly.py (relative error 7.5e-5, below FP16's half-ulp); n added to
// the exponent field as an integer.  x is clamped at -120 first so the
// exponent cannot wrap; 2^-120 is 0 in FP16 and negligible in the FP32 row
// sum, and masked keys (x = -inf) land there too.
// Of every 8 key pairs, these go to the polynomial (a compile-time tuning
// parameter per variant).
#ifndef B200FA_POLY_PAIRS_FP16
#define B200FA_POLY_PAIRS_FP16 1
#endif
#ifndef B200FA_POLY_PAIRS_FP32
#define B200FA_POLY_PAIRS_FP32 1
#endif
template <int kVariant>
constexpr int kPolyPairsOf = kVariant == 0 ? B200FA_POLY_PAIRS_FP16 : B200FA_POLY_PAIRS_FP32;
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
  CUtensorMap tm_q;  // (128, Nq, B*Hq)  fp16, box (64, 128, 1), 128-B swizzle
  CUtensorMap tm_k;  // (128, Nk, B*Hkv)       box (64, 64, 1)
  CUtensorMap tm_v;  // (128, Nk, B*Hkv)       box (64, 128, 1)
  CUtensorMap tm_o;  // (128, Nq, B*Hq)        box (64, 128, 1)
  int32_t Hq, Hkv, group;   // group = Hq / Hkv
  int32_t nqb;              // ceil(Nq / 128)
  int32_t n_kv;             // ceil(Nk / kBlockN)
  int32_t nk_tail;          // valid keys of the last KV block, 1..kBlockN
  int32_t unit_begin, unit_end;
  int32_t num_items;
  float scale_log2;         // scale * log2(e)
  uint32_t flags;
  uint64_t timeout_ns;
  uint32_t* ws;             // status header + trace records
  float* capture;           // capture kernels: [4][heads][n_kv][nq] + [heads][n_kv][nq][128] FP32
  int32_t heads;            // B * Hq
  int32_t nq;               // query rows per head
};

constexpr uint32_t kFlagTrace = 1u;
constexpr uint32_t kFlagTestWithholdP = 2u;
constexpr uint32_t kFlagTimeline = 4u;
constexpr uint32_t kFlagCapture = 8u;
constexpr uint32_t kFlagTestBounds = 16u;  // checking build: one planted out-of-range coordinate
constexpr uint32_t kFlagCausal = 32u;      // causal mask (kernels of the causal translation unit)

// Checking build (B200FA_DEBUG): coordinates, indices and layout are
// verified before use and the roles' block counts at exit; a violation is
// recorded as one of these status codes and takes the abort path.
#ifdef B200FA_DEBUG
constexpr bool kDebug = true;
#else
constexpr bool kDebug = false;
#endif
constexpr uint32_t kDevTimeout = 1u;
constexpr uint32_t kDevBounds = 2u;
constexpr uint32_t kDevPhase = 3u;
constexpr uint32_t kCheckSite = 0x80u;  // low byte of a check's site: 0x80 + check number

// Debug timeline (kFlagTimeline): both CTAs of the first pair stamp
// clock64() at fixed points of their first work item's first kTimelineBlocks
// key blocks.  Layout: u64 [rank][role][block][event] at byte
// kTimelineOffset of the workspace; roles 0-7 = softmax warps 0-7 (lane 0;
// each group's warps stamp the group's blocks), 8 = rank 0's issuers / rank
// 1's forwarder, 9 = TMA thread.  Softmax events: 0 block started, 7 scores
// ready, 1 their loads issued and the reference seen, 2 scores loaded and
// maximum reduced, 3 reference published, 4 exponentials done, 5 P stored
// in TMEM, 6 "P full" arrived.  Issuer events: 0/1 PV
// started/issued, 2/3 S started/issued, 4 "S free" seen; rank 0's warp 11
// (idle otherwise) watches the products complete: 5/6 "S full" / "PV done"
// seen; forwarder events (rank 1): 5/6 K/V forwarded.  TMA events: 0/1 K
// wait/issue, 2/3 V wait/issue.
// The stamps are compiled into the checking build (and any build defining
// B200FA_TIMELINE) only: the product kernels carry no timeline code.
#if defined(B200FA_DEBUG) || defined(B200FA_TIMELINE)
constexpr bool kTimeline = true;
#else
constexpr bool kTimeline = false;
#endif
constexpr int kTimelineRoles = 10;
constexpr int kTimelineBlocks = 48;
constexpr uint32_t kTimelineOffset = 256u + 32u * 1024u;

// The recorder keeps one predicate; the address is recomputed from the
// kernel parameters at each stamp, so a role's loop holds no pointer for it.
struct Timeline {
  const FwdParams* p;
  bool on;
  __device__ __forceinline__ void mark(int role, int j, int e) const {
    if (kTimeline && on && j < kTimelineBlocks) {
      uint64_t* base = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(p->ws) + kTimelineOffset) +
                       cluster_rank() * (uint32_t(kTimelineRoles) * kTimelineBlocks * 8u);
      base[(role * kTimelineBlocks + j) * 8 + e] = clock64();
    }
  }
};

__device__ __forceinline__ Timeline make_timeline(const FwdParams& p, int it, bool thread = true) {
  return Timeline{&p, kTimeline && thread && (p.flags & kFlagTimeline) != 0 && cluster_id_x() == 0 && it == 0};
}

template <typename I>
__host__ __device__ __forceinline__ I ceil_div(I a, I b) {
  return (a + b - 1) / b;
}

// Work items of the unit range [ub, ue): runs of up to kItemUnits
// consecutive units inside one head.  Closed form over (first partial head,
// full heads, last partial head) so that host and device agree without a
// table.
template <typename I>
__host__ __device__ inline I plan_count(I nqb, I ub, I ue) {
  if (ue <= ub) return 0;
  const I G = kItemUnits;
  const I h0 = ub / nqb, h1 = (ue - 1) / nqb;
  const I hi0 = (ue < (h0 + 1) * nqb) ? ue : (h0 + 1) * nqb;
  I n = ceil_div<I>(hi0 - ub, G);
  if (h1 > h0) n += (h1 - h0 - 1) * ceil_div<I>(nqb, G) + ceil_div<I>(ue - h1 * nqb, G);
  return n;
}

template <typename I>
__host__ __device__ inline void plan_decode(I nqb, I ub, I ue, I x, I& bh, I& qb, I& cnt) {
  const I G = kItemUnits;
  const I h0 = ub / nqb, h1 = (ue - 1) / nqb;
  const I hi0 = (ue < (h0 + 1) * nqb) ? ue : (h0 + 1) * nqb;
  const I i0 = ceil_div<I>(hi0 - ub, G);
  if (x < i0) {
    bh = h0;
    qb = ub - h0 * nqb + G * x;
    const I left = hi0 - h0 * nqb - qb;
    cnt = left < G ? left : G;
    return;
  }
  x -= i0;
  const I per = ceil_div<I>(nqb, G);
  const I mid = h1 - h0 - 1;
  if (x < mid * per) {
    bh = h0 + 1 + x / per;
    qb = G * (x % per);
    const I left = nqb - qb;
    cnt = left < G ? left : G;
    return;
  }
  x -= mid * per;
  bh = h1;
  qb = G * x;
  const I left = ue - h1 * nqb - qb;
  cnt = left < G ? left : G;
}

#if B200FA_CAUSAL
// Key blocks of work item `item` with the causal mask: up to the diagonal
// block of the item's last unit.  Every role derives its block count, and
// with it every barrier parity, from this function.
__device__ __forceinline__ int item_blocks_causal(const FwdParams& p, int item) {
  int bh, qb, cnt;
  plan_decode<int>(p.nqb, p.unit_begin, p.unit_end, item, bh, qb, cnt);
  return qb + cnt < p.n_kv ? qb + cnt : p.n_kv;
}
#endif

// Bounded mbarrier waits.  `site` identifies the wait in the status word:
// (rank << 16) | (warp << 8) | barrier slot (or kCheckSite + check number).
struct Waiter {
  uint32_t abort_slot;   // shared u32, nonzero once any thread of the pair gave up
  const FwdParams* p;    // the kernel parameters: bound, status words (read in place)

  __device__ __forceinline__ void fail(uint32_t site, uint32_t code = kDevTimeout) const {
    st_volatile_shared(abort_slot, 1u);
    st_cluster_u32(map_shared(abort_slot, cluster_rank() ^ 1u), 1u);  // the other CTA's flag
    if (atomicCAS(&p->ws[0], 0u, code) == 0u) {
      p->ws[1] = site;
      p->ws[2] = blockIdx.x;
    }
    __threadfence();
  }

  template <bool kCluster>
  __device__ __forceinline__ bool test(uint32_t bar, uint32_t parity) const {
    return kCluster ? mbar_test_cluster(bar, parity) : mbar_test(bar, parity);
  }

  // kCluster: the barrier also receives arrivals from the other CTA.
  template <bool kCluster = false>
  __device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity, uint32_t site) const {
    if (test<kCluster>(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
#pragma unroll 1
      for (int i = 0; i < 16; ++i)
        if (test<kCluster>(bar, parity)) return true;
      if (ld_volatile_shared(abort_slot) != 0u) return false;
      if (global_timer_ns() - t0 > p->timeout_ns) {
        fail(site);
        return false;
      }
    }
  }

  // Checking build: false (after recording B200FA_DEV_BOUNDS with `site`
  // and raising the abort flags) when `ok` is false; the product build
  // compiles the check away.
  __device__ __forceinline__ bool check(bool ok, uint32_t site) const {
    if constexpr (kDebug) {
      if (!ok) fail(site, kDevBounds);
      return ok;
    } else {
      return true;
    }
  }

  // Exit-path wait for work this thread already issued (copies, MMAs); it
  // ignores the abort flag and gives up after `limit_ns`.
  __device__ __forceinline__ void drain(uint32_t bar, uint32_t parity, uint64_t limit_ns) const {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_test_cluster(bar, parity)) {
      if (global_timer_ns() - t0 > limit_ns) return;
    }
  }
};

struct Smem {
  uint32_t base;  // shared-window address of the aligned base
  __device__ __forceinline__ uint32_t bar(int i) const { return base + kSmemBar + 8 * i; }
  __device__ __forceinline__ uint32_t q(int t) const { return base + kSmemQ + t * kQTileBytes; }
  __device__ __forceinline__ uint32_t k(uint32_t e) const { return base + kSmemK + e * kStageBytes; }
  __device__ __forceinline__ uint32_t v(uint32_t e) const { return base + kSmemV + e * kStageBytes; }
  __device__ __forceinline__ uint32_t xchg(uint32_t slot, int row) const {
    return base + kSmemXchg + (slot * kBlockM + uint32_t(row)) * 4u;
  }
  __device__ __forceinline__ uint32_t tmem_slot() const { return base + kSmemMisc; }
  __device__ __forceinline__ uint32_t abort_slot() const { return base + kSmemMisc + 4; }
  // Checking build: key blocks counted by role r (0 S issuer, 1 PV issuer,
  // 2 producer, 3 forwarder, 4/5 softmax group 0/1) at exit.
  __device__ __forceinline__ uint32_t count_slot(int r) const { return base + kSmemMisc + 8 + 4 * r; }
  // Trace: the kernel's start time (two u32 words).
  __device__ __forceinline__ uint32_t start_slot() const { return base + kSmemMisc + 32; }
};

// The CTA counts its key blocks over all its items: block g has its K in K
// ring entry g % kRing, its V in V ring entry g % kRing (the (g / kRing)-th
// use of each), its scores in S buffer g % 2 and its P in P buffer g % 2.
__device__ __forceinline__ uint32_t ring_entry(uint32_t g) { return g % kRing; }
__device__ __forceinline__ uint32_t ring_parity(uint32_t g) { return (g / kRing) & 1u; }
__device__ __forceinline__ uint32_t buf(uint32_t g) { return g & 1u; }
__device__ __forceinline__ uint32_t buf_parity(uint32_t g) { return (g >> 1) & 1u; }

// S = Q K^T over the 128 head dims (8 K=16 steps).  A = Q (two 64-column
// halves kQHalfBytes apart), B = a K stage (two 64-column boxes kKBoxBytes
// apart); step kk starts at half kk/4, 32 bytes per step within a half.
__device__ __forceinline__ void issue_s(uint32_t d_tmem, uint64_t q_desc, uint64_t k_desc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint64_t a = q_desc + uint64_t((kk >> 2) * (kQHalfBytes >> 4) + (kk & 3) * 2);
    const uint64_t b = k_desc + uint64_t((kk >> 2) * (kKBoxBytes >> 4) + (kk & 3) * 2);
    mma_pair_ss(d_tmem, a, b, kIdescQK, kk > 0 ? 1u : 0u);
  }
}

// O (+)= P V over the block's 128 keys (8 K=16 steps): A = P from TMEM (8
// columns per step), B = a V stage (MN-major, 16 keys = 2 KiB per step).
// acc = 0 overwrites O with the first step.
__device__ __forceinline__ void issue_pv(uint32_t o_tmem, uint32_t p_tmem, uint64_t v_desc, uint32_t acc) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    mma_pair_ts(o_tmem, p_tmem + 8u * uint32_t(kk), v_desc + uint64_t(kk * 128), kIdescPV, kk > 0 ? 1u : acc);
}

// ------------------------------------------------------------------ roles
// Rank 0, one thread: every S = Q K^T product of the pair, block by block,
// into S buffer g % 2 once the softmax has read block g - 2's scores from it.
// After each product it commits "S full" on the buffer and the release of
// the block's K stage, both multicast to the two CTAs.
__device__ void s_issuer_role(const FwdParams& p, const Smem& sm, uint32_t tmem_base, const Waiter& w) {
  const uint32_t site = uint32_t(kSIssuerWarp) << 8;
  const int n = p.n_kv;
  uint32_t g = 0;  // the CTA's key blocks so far
  bool ok = true;
  for (int item = int(cluster_id_x()), it = 0; ok && item < p.num_items; item += int(num_clusters_x()), ++it) {
#if B200FA_CAUSAL
    const int n = item_blocks_causal(p, item);  // this item's blocks
#endif
    const Timeline tl = make_timeline(p, it);
    const int qt = it & 1;
    const uint64_t q_desc = smem_desc(sm.q(qt));
    if (!w.wait(sm.bar(kBarQFull + qt), uint32_t(it >> 1) & 1u, site | uint32_t(kBarQFull + qt))) break;
    for (int j = 0; j < n; ++j, ++g) {
      const uint32_t b = buf(g), e = ring_entry(g);
      if (g >= 2 && !w.wait(sm.bar(kBarSFree + int(b)), buf_parity(g - 2u), site | uint32_t(kBarSFree + int(b)))) {
        ok = false;
        break;
      }
      tl.mark(8, j, 4);
      if (!w.wait(sm.bar(kBarKFull + int(e)), ring_parity(g), site | uint32_t(kBarKFull + int(e)))) {
        ok = false;
        break;
      }
      tl.mark(8, j, 2);
      tc_fence_after();
      issue_s(tmem_base + kTmemS + 128u * b, q_desc, smem_desc(sm.k(e)));
      mma_commit_pair_both(sm.bar(kBarSFull + int(b)));
      mma_commit_pair_both(sm.bar(kBarKEmpty + int(e)));
      tl.mark(8, j, 3);
    }
  }
  if constexpr (kDebug) st_volatile_shared(sm.count_slot(0), g);
  // All MMAs this thread issued must be complete before TMEM is freed.
  mma_commit_pair(sm.bar(kBarDrain + 0));
  w.drain(sm.bar(kBarDrain + 0), 0u, 100000000ull);
}

// Rank 0, one thread: every O += P V product of the pair, in block order
// (so O accumulates in order and the item's first product, which overwrites
// O, comes first).  After PV of block g it commits "PV done" on P buffer
// g % 2 (the buffer may be rewritten, and O holds every block up to g) and
// the release of the block's V stage.
__device__ void pv_issuer_role(const FwdParams& p, const Smem& sm, uint32_t tmem_base, const Waiter& w) {
  const uint32_t site = uint32_t(kPVIssuerWarp) << 8;
  const int n = p.n_kv;
  uint32_t g = 0;
  bool ok = true;
  for (int item = int(cluster_id_x()), it = 0; ok && item < p.num_items; item += int(num_clusters_x()), ++it) {
#if B200FA_CAUSAL
    const int n = item_blocks_causal(p, item);  // this item's blocks
#endif
    const Timeline tl = make_timeline(p, it);
    for (int j = 0; j < n; ++j, ++g) {
      const uint32_t b = buf(g), e = ring_entry(g);
      if (!w.wait(sm.bar(kBarVFull + int(e)), ring_parity(g), site | uint32_t(kBarVFull + int(e)))) {
        ok = false;
        break;
      }
      if (!w.wait(sm.bar(kBarPFull + int(b)), buf_parity(g), site | uint32_t(kBarPFull + int(b)))) {
        ok = false;
        break;
      }
      tl.mark(8, j, 0);
      tc_fence_after();
      issue_pv(tmem_base + kTmemO, tmem_base + kTmemP + 64u * b, smem_desc(sm.v(e)), j > 0 ? 1u : 0u);
      mma_commit_pair_both(sm.bar(kBarPVDone + int(b)));
      mma_commit_pair_both(sm.bar(kBarVEmpty + int(e)));
      tl.mark(8, j, 1);
    }
  }
  if constexpr (kDebug) st_volatile_shared(sm.count_slot(1), g);
  mma_commit_pair(sm.bar(kBarDrain + 1));
  w.drain(sm.bar(kBarDrain + 1), 0u, 100000000ull);
}

// Timeline builds, rank 0's otherwise idle warp 11: lane 0 stamps when
// each of the first item's S products completes ("S full"), lane 1 each PV
// product ("PV done").  A buffer's next phase needs the softmax to have
// consumed this one, so a watcher polling without pause sees every phase.
// Observation only: it gives up silently after the bound and never records
// a status.
__device__ void watch_role(const FwdParams& p, const Smem& sm, uint32_t lane) {
  const Timeline tl = make_timeline(p, 0);
  if (!tl.on || cluster_id_x() >= uint32_t(p.num_items) || lane > 1) return;
#if B200FA_CAUSAL
  const int n0 = item_blocks_causal(p, int(cluster_id_x()));
  const int n = n0 < kTimelineBlocks ? n0 : kTimelineBlocks;
#else
  const int n = p.n_kv < kTimelineBlocks ? p.n_kv : kTimelineBlocks;
#endif
  const int bar0 = lane == 0 ? kBarSFull : kBarPVDone;
  for (int j = 0; j < n; ++j) {
    const uint32_t g = uint32_t(j);
    const uint64_t t0 = global_timer_ns();
    while (!mbar_test(sm.bar(bar0 + int(buf(g))), buf_parity(g)))
      if (global_timer_ns() - t0 > p.timeout_ns) return;
    tl.mark(8, j, 5 + int(lane));
  }
}

// Rank 1, one thread: replays the producer's sequence and, as each of this
// CTA's stages lands, arrives on the same barrier of rank 0 (whose MMAs read
// both CTAs' halves).  The arrival is relaxed: the stage's bytes are already
// in this CTA's shared memory (this thread observed their completion on the
// local barrier), and a cluster-scope release -- which orders this thread's
// own earlier memory effects, of which there are none to order here -- took
// about a thousand cycles per arrival under load, enough to pace the whole
// pair at one block per two thousand cycles.
__device__ void forward_role(const FwdParams& p, const Smem& sm, const Waiter& w) {
  const uint32_t site = (1u << 16) | (uint32_t(kForwardWarp) << 8);
  const int n = p.n_kv;
  uint32_t g = 0;
  auto forward = [&](int bar, uint32_t parity) -> bool {
    if (!w.wait(sm.bar(bar), parity, site | uint32_t(bar))) return false;
    mbar_arrive_cluster_relaxed(map_shared(sm.bar(bar), 0));
    return true;
  };
  bool ok = true;
  for (int item = int(cluster_id_x()), it = 0; ok && item < p.num_items; item += int(num_clusters_x()), ++it) {
#if B200FA_CAUSAL
    const int n = item_blocks_causal(p, item);  // this item's blocks
#endif
    const Timeline tl = make_timeline(p, it);
    if (!forward(kBarQFull + (it & 1), uint32_t(it >> 1) & 1u)) break;
    for (int j = 0; j < n; ++j, ++g) {
      const int e = int(ring_entry(g));
      if (!forward(kBarKFull + e, ring_parity(g))) { ok = false; break; }
      tl.mark(8, j, 5);
      if (!forward(kBarVFull + e, ring_parity(g))) { ok = false; break; }
      tl.mark(8, j, 6);
    }
  }
  if constexpr (kDebug) st_volatile_shared(sm.count_slot(3), g);
}

// Both ranks, one thread: this CTA's Q tiles and its halves of every K/V
// block, K and V each into their own ring.
__device__ void load_role(const FwdParams& p, const Smem& sm, const Waiter& w, uint32_t rank) {
  const uint32_t site = (rank << 16) | (uint32_t(kLoadWarp) << 8);
  const int n = p.n_kv;
  uint32_t g = 0;
  uint32_t issued = 0;       // bit e / kRing + e: K / V entry e has ever been loaded
  uint32_t last_par = 0;     // the same bits: parity of its last load
  uint32_t q_issued = 0, q_par = 0;
  bool ok = true;
  for (int item = int(cluster_id_x()), it = 0; ok && item < p.num_items; item += int(num_clusters_x()), ++it) {
    int bh, qb, cnt;
    plan_decode<int>(p.nqb, p.unit_begin, p.unit_end, item, bh, qb, cnt);
#if B200FA_CAUSAL
    const int n = qb + cnt < p.n_kv ? qb + cnt : p.n_kv;  // this item's blocks (item_blocks_causal)
#endif
    const int b = bh / p.Hq;
    const int kvh = b * p.Hkv + (bh - b * p.Hq) / p.group;
    // Rank r holds unit r of the item; a one-unit item repeats it in rank 1
    // (computed, not stored).
    const int u = int(rank) < cnt ? int(rank) : cnt - 1;
    const int row0 = (qb + u) * kBlockM;
    const int qt = it & 1;
    const uint32_t qp = uint32_t(it >> 1) & 1u;
    const Timeline tl = make_timeline(p, it);
    const int kv_planes = p.heads / p.group;
    const int row_end = p.nqb * kBlockM, key_end = p.n_kv * kBlockN;
    // The item's plan: a head of the problem, one or two query blocks inside
    // it and inside the unit range, a KV head of the problem.
    if (!w.check(bh >= 0 && bh < p.heads && qb >= 0 && cnt >= 1 && cnt <= kItemUnits && qb + cnt <= p.nqb &&
                     bh * p.nqb + qb >= p.unit_begin && bh * p.nqb + qb + cnt <= p.unit_end && kvh >= 0 &&
                     kvh < kv_planes,
                 site | (kCheckSite + 0u)))
      break;
    if (!w.wait(sm.bar(kBarQEmpty + qt), qp ^ 1u, site | uint32_t(kBarQEmpty + qt))) break;
    // Q rows of the unit (x = 0 / 64: 16-byte aligned columns).
    const int q_row = row0 + ((p.flags & kFlagTestBounds) ? row_end : 0);
    if (!w.check(q_row >= 0 && q_row < row_end && row0 % kBlockM == 0, site | (kCheckSite + 1u))) break;
    mbar_arrive_expect_tx(sm.bar(kBarQFull + qt), kQTileBytes);
    tma_load_3d(sm.q(qt), &p.tm_q, sm.bar(kBarQFull + qt), 0, row0, bh);
    tma_load_3d(sm.q(qt) + kQHalfBytes, &p.tm_q, sm.bar(kBarQFull + qt), 64, row0, bh);
    q_issued |= 1u << qt;
    q_par = (q_par & ~(1u << qt)) | (qp << qt);
    for (int j = 0; j < n; ++j, ++g) {
      const uint32_t e = ring_entry(g);
      const uint32_t ph = ring_parity(g);
      // K: keys [j*128 + 64r, +64), all 128 head-dim columns, as two 64-column
      // boxes, once S of block g - kRing completed.
      tl.mark(9, j, 0);
      if (!w.wait(sm.bar(kBarKEmpty + int(e)), ph ^ 1u, site | (kBarKEmpty + e))) { ok = false; break; }
      tl.mark(9, j, 1);
      const int krow = j * kBlockN + int(rank) * kKBoxRows;
      if (!w.check(krow >= 0 && krow + kKBoxRows <= key_end, site | (kCheckSite + 2u))) { ok = false; break; }
      mbar_arrive_expect_tx(sm.bar(kBarKFull + int(e)), kStageBytes);
      tma_load_3d(sm.k(e), &p.tm_k, sm.bar(kBarKFull + int(e)), 0, krow, kvh);
      tma_load_3d(sm.k(e) + kKBoxBytes, &p.tm_k, sm.bar(kBarKFull + int(e)), 64, krow, kvh);
      issued |= 1u << e;
      last_par = (last_par & ~(1u << e)) | (ph << e);
      // V: keys [j*128, +128), head-dim columns [64r, +64), once PV of block
      // g - kRing completed.
      tl.mark(9, j, 2);
      if (!w.wait(sm.bar(kBarVEmpty + int(e)), ph ^ 1u, site | (kBarVEmpty + e))) { ok = false; break; }
      tl.mark(9, j, 3);
      if (!w.check(j * kBlockN + kBlockN <= key_end && int(rank) * kPairDims + kPairDims <= kHeadDim,
                   site | (kCheckSite + 3u))) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(sm.bar(kBarVFull + int(e)), kStageBytes);
      tma_load_3d(sm.v(e), &p.tm_v, sm.bar(kBarVFull + int(e)), int(rank) * kPairDims, j * kBlockN, kvh);
      issued |= 1u << (kRing + e);
      last_par = (last_par & ~(1u << (kRing + e))) | (ph << (kRing + e));
    }
  }
  if constexpr (kDebug) st_volatile_shared(sm.count_slot(2), g);
  // Copies still in flight must land before the CTA exits (only possible on
  // the abort path; on the normal path rank 0's MMAs consumed every stage).
  if (!ok || ld_volatile_shared(sm.abort_slot()) != 0u) {
    for (int e = 0; e < kRing; ++e) {
      if (issued & (1u << e)) w.drain(sm.bar(kBarKFull + e), (last_par >> e) & 1u, 50000000ull);
      if (issued & (1u << (kRing + e))) w.drain(sm.bar(kBarVFull + e), (last_par >> (kRing + e)) & 1u, 50000000ull);
    }
    for (int t = 0; t < 2; ++t)
      if (q_issued & (1u << t)) w.drain(sm.bar(kBarQFull + t), (q_par >> t) & 1u, 50000000ull);
  }
}

// Exponentials of 16*kGroups keys (8 pairs per group) of one row:
// x = s * scale*log2(e) - m with packed FP32 FMAs; of every 8 pairs the last
// kPoly go through the FMA-pipe polynomial (exp2_poly2) and the rest through
// MUFU (FP32 ex2).  Writes 8*kGroups packed FP16 pairs of P and adds the row
// sum: FP32 variant, the FP32 exponentials into packed FP32 sums (four
// chains, folded into acc0/acc1); FP16 variant, the FP16 P itself into
// packed FP16 sums (four chains; at most 16*kGroups <= 64 terms of <= 2^8,
// far inside FP16 range), carried over to FP32 once per call (hsum).
// FP16 row sum of 64 keys' P (32 packed pairs): four packed-FP16 chains,
// folded and carried over to FP32.
__device__ __forceinline__ float fp16_row_sum64(const uint32_t* pk) {
  uint32_t hc[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) hc[c] = pk[c];
#pragma unroll
  for (int i = 4; i < 32; ++i) hc[i & 3] = hadd2(hc[i & 3], pk[i]);
  return h2_sum_f32(hadd2(hadd2(hc[0], hc[1]), hadd2(hc[2], hc[3])));
}

template <int kVariant, int kPoly, int kGroups, bool kSum = true>
__device__ __forceinline__ void exp_keys(const uint32_t* r, uint64_t sl2x2, uint64_t nmx2, uint32_t* pk,
                                         uint64_t& acc0, uint64_t& acc1, float& hsum) {
  static_assert(kGroups <= 4, "FP16 partial sums cover at most 64 keys");
  uint64_t cacc[4] = {0ull, 0ull, 0ull, 0ull};
  uint32_t hc[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int g = 0; g < kGroups; ++g) {
#pragma unroll
    for (int pp = 0; pp < 8; ++pp) {
      const int i = g * 8 + pp;  // key pair index
      const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), sl2x2, nmx2);
      uint64_t p2;
      if (pp >= 8 - kPoly) {
        p2 = exp2_poly2(x2);
      } else {
        float a, b;
        f2_unpack(x2, a, b);
        p2 = f2_pack(ex2_approx(a), ex2_approx(b));
      }
      float ea, eb;
      f2_unpack(p2, ea, eb);
      pk[i] = pack_h2(ea, eb);
      if constexpr (kVariant == 1) cacc[pp & 3] = f2_add(cacc[pp & 3], p2);
      if constexpr (kVariant == 0 && kSum) hc[pp & 3] = (g == 0 && pp < 4) ? pk[i] : hadd2(hc[pp & 3], pk[i]);
    }
  }
  if constexpr (kVariant == 0 && kSum) hsum += h2_sum_f32(hadd2(hadd2(hc[0], hc[1]), hadd2(hc[2], hc[3])));
  if constexpr (kVariant == 1) {
    acc0 = f2_add(acc0, f2_add(cacc[0], cacc[2]));
    acc1 = f2_add(acc1, f2_add(cacc[1], cacc[3]));
  }
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

// Keys at or beyond `valid` (the last block's key count) of 64 scores that
// start at key `first` get score -inf.
__device__ __forceinline__ void mask_keys64(uint32_t* r, int first, int valid) {
#pragma unroll
  for (int i = 0; i < 64; ++i)
    if (first + i >= valid) r[i] = __float_as_uint(-INFINITY);
}

// O row of this thread (128 FP32 columns in TMEM) times `f`, in place.
__device__ __forceinline__ void scale_o_row(uint32_t tO, float f) {
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t o[32];
    tmem_ld32(tO + 32u * uint32_t(c), o);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
    tmem_st32(tO + 32u * uint32_t(c), o);
  }
  tmem_wait_st();
}

// Softmax of the CTA's query unit: group grp (warps 4*grp .. 4*grp+3) takes
// the item's key blocks j with j % 2 == grp, one thread per query row (its
// TMEM lane), in both CTAs.  kCapture: the debug-capture instantiation
// (separate kernels, so the production ones carry no capture code).
template <int kVariant, bool kCapture>  // kVariant 0 = FP16 softmax, 1 = FP32 softmax
__device__ void softmax_role(const FwdParams& p, const Smem& sm, uint32_t tmem_base, const Waiter& w,
                             uint32_t warp, uint32_t lane, uint32_t rank) {
  const int grp = int(warp >> 2);  // block parity this group takes
  const int wq = int(warp & 3);    // TMEM lane quarter of this warp
  const int row = wq * 32 + int(lane);
  const uint32_t lane_off = uint32_t(wq * 32) << 16;
  const uint32_t tO = tmem_base + lane_off + kTmemO;
  const uint32_t site = (rank << 16) | (warp << 8);
  const float sl2 = p.scale_log2;
  const uint64_t sl2x2 = f2_pack(sl2, sl2);
  const int n = p.n_kv;
  const bool withhold = (p.flags & kFlagTestWithholdP) != 0 && grp == 1;
  constexpr int kPoly = kPolyPairsOf<kVariant>;
  // "S free" and "P full" live in rank 0; each warp arrives once (lane 0),
  // after its TMEM reads / writes completed (tcgen05.wait::ld / ::st), so
  // rank 1's remote arrival can be relaxed.
  auto arrive_rank0 = [&](int bar) {
    __syncwarp();
    if (lane == 0) {
      if (rank == 0) mbar_arrive(sm.bar(bar));
      else mbar_arrive_cluster_relaxed(map_shared(sm.bar(bar), 0));
    }
  };
  auto arrive_local = [&](int bar) {
    __syncwarp();
    if (lane == 0) mbar_arrive(sm.bar(bar));
  };
  // Bounded wait with a warp-uniform outcome: the warp leaves together, so no
  // warp-collective instruction (tcgen05.ld/st, __syncwarp) ever runs with
  // part of the warp gone.
  auto wait_warp = [&](int bar, uint32_t parity) -> bool {
    return __all_sync(0xffffffffu, w.wait(sm.bar(bar), parity, site | uint32_t(bar)));
  };
  bool ok = true;
  uint32_t blocks_done = 0;  // checking build: this group's key blocks
#if B200FA_CAUSAL
  uint32_t g_items = 0;      // the CTA's key blocks of all earlier items
#endif

  for (int item = int(cluster_id_x()), it = 0; ok && item < p.num_items; item += int(num_clusters_x()), ++it) {
#if B200FA_CAUSAL
    const int n = item_blocks_causal(p, item);  // this item's blocks
    const uint32_t g0 = g_items;                // the CTA's block count before this item
    g_items += uint32_t(n);
    // This thread's query row (rank r holds unit r of the item; a one-unit
    // item repeats it in rank 1): the mask's bound.
    int qrow_g;
    {
      int bh_i, qb_i, cnt_i;
      plan_decode<int>(p.nqb, p.unit_begin, p.unit_end, item, bh_i, qb_i, cnt_i);
      qrow_g = (qb_i + (int(rank) < cnt_i ? int(rank) : cnt_i - 1)) * kBlockM + row;
    }
#else
    const uint32_t g0 = uint32_t(it) * uint32_t(n);  // the CTA's block count before this item
#endif
    float m_cur = -INFINITY;  // reference of this group's last block (log2 domain)
    float l_g = 0.f;          // this group's row sum over its blocks, relative to m_cur
    const Timeline tl = make_timeline(p, it, lane == 0);
    // Debug capture: cap_on (this CTA's unit exists in the item) is
    // warp-uniform, cap_row per thread (its query row exists).  Record
    // (b*Hq+hq, block j, row) sits at index (bh*n + j)*nq + row of each
    // scalar plane (stride heads*n*nq) and, times 128, in the O plane after
    // them.
    bool cap_on = false, cap_row = false;
    size_t cap_idx = 0;
    if constexpr (kCapture) {
      int bh, qb, cnt;
      plan_decode<int>(p.nqb, p.unit_begin, p.unit_end, item, bh, qb, cnt);
      const int qrow = (qb + int(rank)) * kBlockM + row;
      cap_on = int(rank) < cnt;
      cap_row = cap_on && qrow < p.nq;
      cap_idx = (size_t(bh) * size_t(n)) * size_t(p.nq) + size_t(qrow);
    }
    const size_t cap_plane = size_t(p.heads) * size_t(n) * size_t(p.nq);
    // O after PV(jb) (unnormalised FP32, relative to that block's m):
    // read the row from TMEM (whole warp), store it.
    auto capture_o = [&](int jb) {
      float4* orec = reinterpret_cast<float4*>(p.capture + 4 * cap_plane +
                                               (cap_idx + size_t(jb) * size_t(p.nq)) * size_t(kHeadDim));
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tO + 32 * c, o);
        tmem_wait_ld();
        if (cap_row) {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            orec[8 * c + u] = make_float4(__uint_as_float(o[4 * u]), __uint_as_float(o[4 * u + 1]),
                                          __uint_as_float(o[4 * u + 2]), __uint_as_float(o[4 * u + 3]));
        }
      }
    };
    // PV of block gp done (and, one issuer in order, every PV before it).
    // The barrier's next phase is PV of block gp + 2, which cannot complete
    // before this group's next "P full": no phase is missed.
    auto wait_pv = [&](uint32_t gp) -> bool { return wait_warp(kBarPVDone + int(buf(gp)), buf_parity(gp)); };

    for (int j = grp; j < n; j += 2) {
      const uint32_t gb = g0 + uint32_t(j);
      const uint32_t b = buf(gb);
      const uint32_t tS = tmem_base + lane_off + kTmemS + 128u * b;
      const uint32_t tP = tmem_base + lane_off + kTmemP + 64u * b;
      float m_prev = -INFINITY;
      tl.mark(int(warp), j, 0);
      if (!wait_warp(kBarSFull + int(b), buf_parity(gb))) {
        ok = false;
        break;
      }
      tl.mark(int(warp), j, 7);
      tc_fence_after();
#if B200FA_CAUSAL
      // Valid keys of the block for this row: the last block's key count
      // and the keys up to the row.
      int valid = j == p.n_kv - 1 ? p.nk_tail : kBlockN;
      if (qrow_g - j * kBlockN + 1 < valid) valid = qrow_g - j * kBlockN + 1;
      const bool tail = valid < kBlockN;
#else
      const bool tail = (j == n - 1 && p.nk_tail < kBlockN);
#endif
      // The scores: one 128-column load in the FP16 kernel, four 32-column
      // loads in the FP32 kernel (each measured the faster for its kernel).
      uint32_t r[kBlockN];
      if constexpr (kVariant == 0) {
        tmem_ld128(tS, r);
      } else {
        tmem_ld32(tS, r);
        tmem_ld32(tS + 32u, r + 32);
        tmem_ld32(tS + 64u, r + 64);
        tmem_ld32(tS + 96u, r + 96);
      }
      // While the scores are on their way: the reference after block j-1
      // ("ref" gb-1, published by the other group).  Waited for also at an
      // item's first block (value unused): the wait orders this group's
      // write of slot gb % 2 after the other group's read of it.
      if (gb > 0) {
        if (!wait_warp(kBarRef + int((gb - 1u) & 1u), ((gb - 1u) >> 1) & 1u)) {
          tmem_wait_ld();
          ok = false;
          break;
        }
        if (j > 0) m_prev = ld_shared_f32(sm.xchg((gb - 1u) & 1u, row));
      }
      tl.mark(int(warp), j, 1);
      tmem_wait_ld();
      if (tail) {
#if B200FA_CAUSAL
        mask_keys64(r, 0, valid);
        mask_keys64(r + 64, 64, valid);
#else
        mask_keys64(r, 0, p.nk_tail);
        mask_keys64(r + 64, 64, p.nk_tail);
#endif
      }
      arrive_rank0(kBarSFree + int(b));  // the S issuer may refill the buffer
      const float mx = fmaxf(row_max64(r), row_max64(r + 64)) * sl2;
      tl.mark(int(warp), j, 2);
      // This group's partial sum follows the reference the other group left.
      if (j >= 2 && m_prev != m_cur) l_g *= ex2_approx(m_cur - m_prev);
      float m_new = m_prev, alpha = 1.f;
      bool moved = false;
      if (mx > m_prev + kRescaleLog2) {
        m_new = mx;
        moved = j > 0;
        alpha = ex2_approx(m_prev - mx);  // 0 at the item's first block
      }
      st_shared_f32(sm.xchg(gb & 1u, row), m_new);
      arrive_local(kBarRef + int(gb & 1u));
      tl.mark(int(warp), j, 3);
      if constexpr (kCapture) {
        if (cap_on && j > 0) {
          if (!wait_pv(gb - 1u)) { ok = false; break; }
          tc_fence_after();
          capture_o(j - 1);
        }
      }
      if (moved) l_g *= alpha;
      m_cur = m_new;
      uint32_t pk[kBlockN / 2];
      uint64_t acc0 = 0ull, acc1 = 0ull;  // packed FP32 partial row sums
      float hsum = 0.f;                   // FP16 variant: sums of FP16 group sums
      const uint64_t nm = f2_pack(-m_new, -m_new);
      // FP16 variant: the row sum of the FP16 P is taken after P has been
      // handed over (its conversions then long complete, and off the
      // hand-off path); the capture kernels need it earlier.
      constexpr bool kLateSum = kVariant == 0 && !kCapture;
      exp_keys<kVariant, kPoly, 4, !kLateSum>(r, sl2x2, nm, pk, acc0, acc1, hsum);
      exp_keys<kVariant, kPoly, 4, !kLateSum>(r + 64, sl2x2, nm, pk + 32, acc0, acc1, hsum);
      tl.mark(int(warp), j, 4);
      if (__any_sync(0xffffffffu, moved)) {
        // Lazy correction of the running output before this block's P is
        // handed over: PV(gb-1) must be complete (PV(gb) waits for "P full").
        if (!wait_pv(gb - 1u)) { ok = false; break; }
        tc_fence_after();
        scale_o_row(tO, moved ? alpha : 1.f);
      }
      float a0, b0, a1, b1;
      f2_unpack(acc0, a0, b0);
      f2_unpack(acc1, a1, b1);
      const float z = ((a0 + b0) + (a1 + b1)) + hsum;
      if constexpr (!kLateSum) l_g += z;
      if constexpr (kCapture) {
        // Running row sum over both groups: the other group's record of
        // block j-1 holds the total after it; it was written and fenced
        // before that group's "P full", which PV(j-1) -- waited for above --
        // follows.
        if (cap_row) {
          float* rec = p.capture + cap_idx + size_t(j) * size_t(p.nq);
          const float l_prev = j == 0 ? 0.f : ld_volatile_global_f32(rec + cap_plane - p.nq);
          rec[0] = m_new;
          rec[cap_plane] = (j == 0 ? 0.f : alpha * l_prev) + z;
          rec[2 * cap_plane] = j == 0 ? 0.f : alpha;
          rec[3 * cap_plane] = z;
        }
        __threadfence();
      }
      // P buffer b is free once PV of block gb - 2 completed.
      if (gb >= 2 && !wait_pv(gb - 2u)) { ok = false; break; }
      tc_fence_after();
      if constexpr (kVariant == 0) {  // one 64-column store / two 32-column stores, as the loads
        tmem_st64(tP, pk);
      } else {
        tmem_st32(tP, pk);
        tmem_st32(tP + 32u, pk + 32);
      }
      tmem_wait_st();
      tl.mark(int(warp), j, 5);
      tc_fence_before();
      if (!(withhold && it == 0 && j == 1)) arrive_rank0(kBarPFull + int(b));
      if constexpr (kLateSum) l_g += fp16_row_sum64(pk) + fp16_row_sum64(pk + 32);
      ++blocks_done;
      tl.mark(int(warp), j, 6);
    }
    if (!ok) break;

    // ---- epilogue: O / l -> FP16 -> swizzled smem (this item's Q tile) -> TMA store.
    // Group grp converts head-dim columns [64 grp, +64) of its rows.
    const int qt = it & 1;
    const uint32_t sQ = sm.q(qt);
    const uint32_t g_last = g0 + uint32_t(n) - 1u;
    if (!wait_pv(g_last)) { ok = false; break; }  // every PV of the item complete
    tc_fence_after();
    // Both partial sums to the final reference, then added.
    float m_final = m_cur;
    if ((n - 1) % 2 != grp) {
      if (!wait_warp(kBarRef + int(g_last & 1u), (g_last >> 1) & 1u)) {
        ok = false;
        break;
      }
      m_final = ld_shared_f32(sm.xchg(g_last & 1u, row));
    }
    if (l_g != 0.f && m_final != m_cur) l_g *= ex2_approx(m_cur - m_final);
    if constexpr (kCapture) {
      if (cap_on && grp == 0) capture_o(n - 1);
    }
    // Exchange through the two reference slots: phase 0 -- every reference
    // read; group 0 writes slot g_last % 2 (which the other group's next
    // write follows its own read of), group 1 the other; phase 1 -- read.
    arrive_local(kBarXchg);
    if (!wait_warp(kBarXchg, 0u)) { ok = false; break; }
    const uint32_t mine = grp == 0 ? (g_last & 1u) : ((g_last + 1u) & 1u);
    st_shared_f32(sm.xchg(mine, row), l_g);
    arrive_local(kBarXchg);
    if (!wait_warp(kBarXchg, 1u)) { ok = false; break; }
    const float l = l_g + ld_shared_f32(sm.xchg(mine ^ 1u, row));
    const float inv_l = 1.f / l;
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t o[32];
      tmem_ld32(tO + 64u * uint32_t(grp) + 32u * uint32_t(c), o);
      tmem_wait_ld();
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t h0 = pack_h2(__uint_as_float(o[8 * u + 0]) * inv_l, __uint_as_float(o[8 * u + 1]) * inv_l);
        const uint32_t h1 = pack_h2(__uint_as_float(o[8 * u + 2]) * inv_l, __uint_as_float(o[8 * u + 3]) * inv_l);
        const uint32_t h2 = pack_h2(__uint_as_float(o[8 * u + 4]) * inv_l, __uint_as_float(o[8 * u + 5]) * inv_l);
        const uint32_t h3 = pack_h2(__uint_as_float(o[8 * u + 6]) * inv_l, __uint_as_float(o[8 * u + 7]) * inv_l);
        const int gu = 8 * grp + 4 * c + u;  // 16-byte unit of the 256-byte output row
        const uint32_t addr = sQ + uint32_t(gu >> 3) * kQHalfBytes + uint32_t(row) * 128 +
                              (uint32_t((gu & 7) ^ (row & 7)) << 4);
        st_shared_v4(addr, h0, h1, h2, h3);
      }
    }
    tc_fence_before();
    fence_proxy_async_smem();
    arrive_local(kBarOStaged);
    if (warp == 0 && lane == 0) {
      int bh, qb, cnt;
      plan_decode<int>(p.nqb, p.unit_begin, p.unit_end, item, bh, qb, cnt);
      const int orow = (qb + int(rank)) * kBlockM;
      if (!w.wait(sm.bar(kBarOStaged), uint32_t(it) & 1u, site | kBarOStaged)) {
        ok = false;
      } else if (int(rank) < cnt &&
                 !w.check(orow >= 0 && orow < p.nqb * kBlockM && bh >= 0 && bh < p.heads, site | (kCheckSite + 4u))) {
        ok = false;
      } else {
        if (int(rank) < cnt) {
          tma_store_3d(&p.tm_o, sQ, 0, orow, bh);
          tma_store_3d(&p.tm_o, sQ + kQHalfBytes, 64, orow, bh);
          bulk_commit_group();
          bulk_wait_group_read0();
        }
        mbar_arrive(sm.bar(kBarQEmpty + qt));
      }
    }
    // A failure seen by warp 0's storing lane ends the loop for its whole warp.
    ok = __all_sync(0xffffffffu, ok);
  }
  if (warp == 0 && lane == 0) bulk_wait_group0();
  if constexpr (kDebug) {
    if (wq == 0 && lane == 0) st_volatile_shared(sm.count_slot(4 + grp), blocks_done);
  }
}

__device__ __forceinline__ Smem smem_of(uint8_t* smem_raw) { return Smem{(smem_addr(smem_raw) + 1023u) & ~1023u}; }

__device__ __forceinline__ Waiter waiter_of(const FwdParams& p, const Smem& sm) { return Waiter{sm.abort_slot(), &p}; }

// The kernel runs in three phases -- setup, roles, teardown -- that share no
// register: what a later phase needs is read again from special registers
// or shared memory.  Nothing is then live across the role split, where the
// warpgroups' register counts differ (a value live there is spilled).
__device__ __forceinline__ void setup_phase(const FwdParams& p, uint8_t* smem_raw) {
  const Smem sm = smem_of(smem_raw);
  const uint32_t tid = tid_x();
  const uint32_t warp = tid >> 5, lane = tid & 31u;
  const uint32_t rank = cluster_rank();
  if (tid == 0) {
    const uint32_t fed = rank == 0 ? 2u : 1u;  // rank 0's full barriers also count rank 1's forward
    for (int t = 0; t < 2; ++t) {
      mbar_init(sm.bar(kBarQFull + t), fed);
      mbar_init(sm.bar(kBarQEmpty + t), 1);
      mbar_init(sm.bar(kBarSFull + t), 1);
      mbar_init(sm.bar(kBarSFree + t), kGroupWarps);
      mbar_init(sm.bar(kBarPFull + t), kGroupWarps);
      mbar_init(sm.bar(kBarPVDone + t), 1);
      mbar_init(sm.bar(kBarRef + t), 4);
      mbar_init(sm.bar(kBarDrain + t), 1);
    }
    mbar_init(sm.bar(kBarXchg), 8);
    mbar_init(sm.bar(kBarOStaged), 8);
    for (int e = 0; e < kRing; ++e) {
      mbar_init(sm.bar(kBarKFull + e), fed);
      mbar_init(sm.bar(kBarKEmpty + e), 1);
      mbar_init(sm.bar(kBarVFull + e), fed);
      mbar_init(sm.bar(kBarVEmpty + e), 1);
    }
    st_volatile_shared(sm.abort_slot(), 0u);
    for (int r = 0; r < 6; ++r) st_volatile_shared(sm.count_slot(r), 0u);
    fence_mbarrier_init();
  }
  if (warp == kLoadWarp && lane == 0) {
    const uint64_t t_start = global_timer_ns();
    st_volatile_shared(sm.start_slot(), uint32_t(t_start));
    st_volatile_shared(sm.start_slot() + 4, uint32_t(t_start >> 32));
    tma_prefetch_map(&p.tm_q);
    tma_prefetch_map(&p.tm_k);
    tma_prefetch_map(&p.tm_v);
    tma_prefetch_map(&p.tm_o);
  }
  if (warp == 0) {
    tmem_alloc_pair(sm.tmem_slot(), kTmemCols);
    tmem_relinquish_pair();
  }
  // Barriers of both CTAs initialised and TMEM allocated before any
  // cross-CTA arrival or pair MMA.
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if constexpr (kDebug) {
    // The whole 512-column allocation starts at lane 0, column 0, and the
    // aligned layout ends inside the dynamic shared memory.
    if (tid == 0) {
      const uint32_t tmem_base = ld_volatile_shared(sm.tmem_slot());
      waiter_of(p, sm).check(tmem_base == 0u && sm.base + uint32_t(kSmemUsed) <= smem_addr(smem_raw) + uint32_t(kSmemBytes),
                             (rank << 16) | (kCheckSite + 5u));
    }
  }
}

template <int kVariant, bool kCapture>
__device__ __forceinline__ void role_phase(const FwdParams& p, uint8_t* smem_raw) {
  const Smem sm = smem_of(smem_raw);
  const uint32_t tid = tid_x();
  const uint32_t warp = tid >> 5, lane = tid & 31u;
  if (warp < 8) {
    regs_increase<kSoftmaxRegs>();
    const uint32_t tmem_base = ld_volatile_shared(sm.tmem_slot());
    softmax_role<kVariant, kCapture>(p, sm, tmem_base, waiter_of(p, sm), warp, lane, cluster_rank());
  } else {
    regs_decrease<kControlRegs>();
    const uint32_t rank = cluster_rank();
    if (lane == 0) {
      const uint32_t tmem_base = ld_volatile_shared(sm.tmem_slot());
      const Waiter w = waiter_of(p, sm);
      if (rank == 0 && warp == kSIssuerWarp) s_issuer_role(p, sm, tmem_base, w);
      else if (rank == 0 && warp == kPVIssuerWarp) pv_issuer_role(p, sm, tmem_base, w);
      else if (warp == kLoadWarp) load_role(p, sm, w, rank);
      else if (rank == 1 && warp == kForwardWarp) forward_role(p, sm, w);
    }
    if (kTimeline && rank == 0 && warp == kForwardWarp) watch_role(p, sm, lane);
  }
  __syncwarp();
}

__device__ __forceinline__ void teardown_phase(const FwdParams& p, uint8_t* smem_raw) {
  const Smem sm = smem_of(smem_raw);
  const uint32_t tid = tid_x();
  const uint32_t warp = tid >> 5;
  const uint32_t rank = cluster_rank();
  // Rank 0's MMAs read and write both CTAs' memories: neither CTA frees
  // TMEM or leaves before the pair is done.
  tc_fence_before();
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(ld_volatile_shared(sm.tmem_slot()), kTmemCols);
  }
  if constexpr (kDebug) {
    // Every role counted the same key blocks: the parity of every mbarrier
    // wait derives from those counts.
    if (tid == 0 && ld_volatile_shared(sm.abort_slot()) == 0u) {
      uint32_t items = 0;
      for (int item = int(cluster_id_x()); item < p.num_items; item += int(num_clusters_x())) ++items;
#if B200FA_CAUSAL
      uint32_t want = 0;
      for (int item = int(cluster_id_x()); item < p.num_items; item += int(num_clusters_x()))
        want += uint32_t(item_blocks_causal(p, item));
      (void)items;
#else
      const uint32_t want = items * uint32_t(p.n_kv);
#endif
      const uint32_t groups = ld_volatile_shared(sm.count_slot(4)) + ld_volatile_shared(sm.count_slot(5));
      bool same = ld_volatile_shared(sm.count_slot(2)) == want && groups == want;
      if (rank == 0) same = same && ld_volatile_shared(sm.count_slot(0)) == want && ld_volatile_shared(sm.count_slot(1)) == want;
      else same = same && ld_volatile_shared(sm.count_slot(3)) == want;
      if (!same) waiter_of(p, sm).fail((rank << 16) | (kCheckSite + 6u), kDevPhase);
    }
  }
  if ((p.flags & kFlagTrace) && tid == kLoadWarp * 32 && blockIdx.x < 1024) {
    uint32_t* rec = p.ws + (256 + 32 * blockIdx.x) / 4;
    int items = 0;
    for (int item = int(cluster_id_x()); item < p.num_items; item += int(num_clusters_x())) ++items;
    const uint64_t t_end = global_timer_ns();
    rec[0] = sm_id();
    rec[1] = uint32_t(items);
    rec[2] = ld_volatile_shared(sm.start_slot());
    rec[3] = ld_volatile_shared(sm.start_slot() + 4);
    rec[4] = uint32_t(t_end);
    rec[5] = uint32_t(t_end >> 32);
    rec[6] = rank;
    rec[7] = 0u;
  }
}

template <int kVariant, bool kCapture>
__device__ __forceinline__ void attention_fwd_body(const FwdParams& p) {
  extern __shared__ uint8_t smem_raw[];
  setup_phase(p, smem_raw);
  role_phase<kVariant, kCapture>(p, smem_raw);
  teardown_phase(p, smem_raw);
}

}  // namespace b200fa
