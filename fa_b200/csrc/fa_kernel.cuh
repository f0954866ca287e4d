// fa_kernel.cuh -- the sm_100a warp-specialised flash-attention forward.
//
// Operator (reference semantics: backends/npu_fa/backend.py:36-49, FP32
// formula backends/expert_v2/impl_tl.py:701-717):
//   O[b,h] = softmax(Q[b,h] K[b,kv]^T * scale) V[b,kv],  kv = b*Hkv + h/(Hq/Hkv)
// (GQA head map of panel_kernel.h:274), non-causal, D = 128, FP16 in/out.
//
// Work decomposition.  A work unit is one 128-row query block of one (b, hq),
// linearised ((b*Hq)+hq)*ceil(Nq/128)+qb (cce_task.h:28-35 order).  A work
// item is up to four consecutive units of the same head (512 query rows)
// that share every K/V block.  Items are dealt round-robin to a persistent
// grid of CTA pairs (clusters of two CTAs on the two SMs of a TPC), one pair
// per TPC.
//
// The pair.  Both tensor-core products run as pair MMAs (tcgen05
// cta_group::2, M = 256) issued by rank 0: each CTA holds 128 query rows of
// a tile, and the B operand is split between the two shared memories --
// rank r holds keys [64r, 64r+64) of every 128-key K block (S = Q K^T) and
// head-dim columns [64r, 64r+64) of every V block (O = P V).  Per SM and
// K=16 step the QK product then reads 4 KiB of Q and 2 KiB of K from shared
// memory (48 cycles at 128 B/clk against 64 cycles of tensor work), and each
// SM loads only half of every K/V block.
//
// CTA roles (384 threads = 3 warpgroups), the same in both CTAs:
//   warps 0-3   softmax, query tile 0 (TMEM lanes = rows)
//   warps 4-7   softmax, query tile 1
//   warp  8/10  rank 0: MMA issuer of tile 0 / tile 1 (one thread each)
//   warp  9     TMA producer (one thread): this CTA's Q tiles and K/V halves
//   warp  11    rank 1: forwards its TMA completions to rank 0's barriers
// Unit u = 2t + r of an item is tile t of rank r.
//
// One issuer thread per tile: a thread that has tcgen05.mma in flight
// stalls on its next shared-memory access (an mbarrier probe included)
// until those MMAs drain, so a single issuer that waits between products
// leaves the tensor pipe idle.  With one issuer per tile, one tile's
// products keep the pipe busy while the other tile's issuer waits.
//
// Tensor memory, per tile t (same columns in both CTAs):
//   S_t [128t, 128t+128)     FP32 scores of the current 128-key block, as
//                            two halves: keys 0-63 in columns [0,64), keys
//                            64-127 in [64,128).  Once the softmax has read
//                            them, P_t (FP16 pairs) takes columns [96,128)
//                            (keys 0-63) and [64,96) (keys 64-127)
//   O_t [256+128t, +128)     FP32 output accumulator
//
// Shared memory (1024-B aligned, 128-byte swizzle as the TMA writes it):
//   Q0, Q1 (2 x 32 KiB: two 64-column halves of 128 rows; each also stages
//   its tile's FP16 output for the TMA store), a ring of kStages 16 KiB
//   stages holding this CTA's part of K_j (32 keys of each S half, as two
//   64-column boxes of 32 rows per half) and of V_j (one box of 128 rows x
//   64 columns) alternately, mbarriers.
//
// Per key block j the issuer of tile t works in two windows.  After "P
// half" j (all 8 softmax warps of the tile, 4 per CTA, have read S_t(j) and
// written P_t(j) keys 0-63): S_t(j+1) keys 0-63 ("S low" j+1, its columns
// hold no P), then PV over keys 0-63.  After "P full" j (keys 64-127
// written): PV over keys 64-127, then S_t(j+1) keys 64-127 ("S high" j+1)
// over the columns both PV halves read -- one thread issues them, and the
// tensor pipe executes its products in order.  So S_t(j+1) keys 0-63 are
// computed while the softmax still works on block j, and the ordering gives
// the softmax its guarantees without further waits: "S high" j+1 means the
// PV of block j is complete, so O_t may be rescaled and P_t(j+1) written.
// Splitting S costs shared-memory bandwidth (an N = 64 half reads Q once
// per 32 tensor cycles: 40 cycles at 128 B/clk) and buys S(j+1) keys 0-63
// off the softmax's path.  The softmax releases its use of the K/V ring
// slots locally (K_j once "S high" j, V_j once "S high" j+1 or, for the
// item's last block, "O final"); a slot is refilled after both tiles
// released it.  Rank 1's TMA completions reach rank 0 through its warp 11,
// which waits for each local stage and arrives on rank 0's barrier: no copy
// ever signals the other CTA.
//
// Online softmax (per query row, one thread per row): running reference
// maximum m (log2 domain), running sum l.  The reference moves only when a
// block's maximum exceeds it by more than kRescaleLog2 (lazy rescaling), so
// P <= 2^kRescaleLog2 and O/l is exact at the end whatever the reference.
// When it moves, the warp rescales its 32 rows of O in TMEM.  After a
// tile's first block the exponentials of keys 0-63 are computed against the
// current reference while keys 64-127 are loaded and reduced, and redone in
// the rare block where the reference moves.
//
// Every wait is bounded (global timer); on expiry the kernel records
// B200FA_DEV_TIMEOUT in the workspace, raises the abort flag of both CTAs,
// every role leaves its loop, in-flight copies and MMAs are drained with a
// second bound, TMEM is freed and the kernel returns.
#pragma once
#include <cstdint>
#include <cuda.h>
#include "ptx.cuh"

namespace b200fa {

constexpr int kBlockM = 128;    // query rows per tile (per CTA)
constexpr int kBlockN = 128;    // keys per KV block
constexpr int kHeadDim = 128;   // head dimension (fixed)
constexpr int kPairKeys = kBlockN / 2;    // K rows of a block held by each CTA
constexpr int kPairDims = kHeadDim / 2;   // V head-dim columns held by each CTA
constexpr int kItemUnits = 4;   // query units per work item (2 tiles x 2 CTAs)
constexpr int kStages = 10;     // K/V ring depth (even: a slot only ever holds K or only V)
constexpr int kQTileBytes = kBlockM * kHeadDim * 2;   // 32 KiB
constexpr int kQHalfBytes = kQTileBytes / 2;          // TMA box: 64 cols x 128 rows
constexpr int kKBoxRows = kPairKeys / 2;             // K rows of one S half held by each CTA
constexpr int kKBoxBytes = kKBoxRows * 128;           // TMA box: 64 cols x 32 rows
constexpr int kKPartBytes = 2 * kKBoxBytes;           // one S half's keys, all 128 columns
constexpr int kStageBytes = 2 * kKPartBytes;          // 16 KiB
static_assert(kBlockN * kPairDims * 2 == kStageBytes, "K and V stages must have the same size");
static_assert(kStages % 2 == 0, "ring slots must alternate K and V consistently");
constexpr int kThreads = 384;    // 3 warpgroups
constexpr int kMmaWarp = 8;      // tile t's issuer: warp kMmaWarp + 2t (rank 0)
constexpr int kLoadWarp = 9;
constexpr int kForwardWarp = 11; // rank 1
// Register split (setmaxnreg): launch 384 x 168 = 64512; softmax warpgroups
// 256 x 208 + warpgroup 2 128 x 88 = 64512.
constexpr uint32_t kLaunchRegs = 168;
constexpr uint32_t kSoftmaxRegs = 208;
constexpr uint32_t kControlRegs = 88;
static_assert(256 * kSoftmaxRegs + 128 * kControlRegs <= kThreads * kLaunchRegs, "register split exceeds the launch budget");
constexpr float kRescaleLog2 = 8.0f;  // lazy-rescale threshold (factor 256)

// Tensor memory columns.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;       // + 128 t
constexpr uint32_t kTmemO = 256;     // + 128 t
constexpr uint32_t kTmemPLo = 96;    // column offset within S_t of P for keys 0-63
constexpr uint32_t kTmemPHi = 64;    // column offset within S_t of P for keys 64-127
static_assert(kTmemO + 256 <= kTmemCols, "TMEM budget");

// Barrier slots.  "rank 0" barriers are only waited on in rank 0.
constexpr int kBarQFull = 0;     // [2] Q tile landed (rank 0: own TMA + rank 1's forward; rank 1: own TMA)
constexpr int kBarQEmpty = 2;    // [2] Q buffer free (epilogue store read it)                    local
constexpr int kBarSLo = 4;       // [2] S_t keys 0-63 of a block computed   (pair commit to both CTAs)
constexpr int kBarPHalf = 6;     // [2] rank 0: P_t keys 0-63 written by the 8 softmax warps of tile t
constexpr int kBarPFull = 8;     // [2] rank 0: P_t keys 64-127 written (and O_t rescaled)
constexpr int kBarOStaged = 10;  // [2] O tile staged in smem (128 threads)                       local
constexpr int kBarDrain = 12;    // [2] rank 0: MMA drain of issuer t at exit
constexpr int kBarOFinal = 14;   // [2] last PV_t of an item done   (pair commit to both CTAs)
constexpr int kBarSHi = 16;      // [2] S_t keys 64-127 of a block computed (pair commit to both CTAs)
constexpr int kBarKVFull = 18;   // [kStages] (rank 0: own TMA + rank 1's forward)
constexpr int kBarKVEmpty = kBarKVFull + kStages;  // [kStages] released by both tiles' softmax   local
constexpr int kNumBars = kBarKVEmpty + kStages;
constexpr uint32_t kTileWarps = 8;  // softmax warps per tile in the pair (arrivals on P half / P full)

constexpr int kSmemQ = 0;
constexpr int kSmemKV = 2 * kQTileBytes;
constexpr int kSmemBar = kSmemKV + kStages * kStageBytes;
constexpr int kSmemMisc = kSmemBar + kNumBars * 8;  // TMEM base (4 B), abort flag (4 B)
constexpr int kSmemUsed = kSmemMisc + 16;
constexpr int kSmemBytes = kSmemUsed + 1024;  // + slack for 1024-B alignment
static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");
static_assert(kSmemBar % 8 == 0, "mbarrier alignment");
static_assert(kKBoxBytes % 1024 == 0 && kStageBytes % 1024 == 0, "128-byte swizzle atoms must stay 1024-B aligned");

// tcgen05 instruction descriptors, kind::f16 (PTX ISA "Instruction
// descriptor"): bits 4-5 D format (1 = F32), 7-9 A format (0 = F16),
// 10-12 B format (0 = F16), 15 A major (0 = K), 16 B major (1 = MN),
// 17-22 N>>3, 24-28 M>>4.  M = 256: the pair's rows.
constexpr uint32_t kIdescQK = (1u << 4) | (uint32_t((kBlockN / 2) >> 3) << 17) | (uint32_t(256 >> 4) << 24);
constexpr uint32_t kIdescPV = (1u << 4) | (1u << 16) | (uint32_t(kHeadDim >> 3) << 17) | (uint32_t(256 >> 4) << 24);
static_assert((kBlockN / 2) % 16 == 0 && kBlockN <= 256, "M=256 needs N a multiple of 16");

// Shared-memory matrix descriptors (PTX ISA "Matrix Descriptor"), 128-byte
// swizzle, sm_100 version bit.  Low word: start address >> 4 (bits 0-13),
// leading byte offset >> 4 (bits 16-29).  High word: stride byte offset >> 4
// (bits 0-13), version 1 (bit 14), layout SWIZZLE_128B = 2 (bits 29-31).
// Rows of 128 B, 8-row groups 1024 B apart (SBO) for Q, K (K-major) and V
// (MN-major: rows are keys, 64 head-dim columns per row).  The leading
// offset is unused: swizzled K-major layouts ignore it and each CTA's V
// half is a single 64-column block; it is set to 16 B.
constexpr uint32_t kDescHi = uint32_t(1024 >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint32_t desc_lo(uint32_t saddr) { return ((saddr & 0x3FFFFu) >> 4) | (1u << 16); }

// exp2 on the FMA pipe for two lanes.  Cody-Waite split x = n + f with
// n = round(x) taken from the low mantissa bits of x + 1.5*2^23 and
// f = x - n in [-1/2, 1/2]; 2^f by the degree-3 minimax polynomial of
// fit_exp2_poly.py (relative error 7.5e-5, below FP16's half-ulp); n added to
// the exponent field as an integer.  x is clamped at -120 first so the
// exponent cannot wrap; 2^-120 is 0 in FP16 and negligible in the FP32 row
// sum, and masked keys (x = -inf) land there too.
// Of every 8 key pairs, these go to the polynomial (measured per variant:
// the FP32 variant's packed FP32 sums already load the FMA pipe).
template <int kVariant>
constexpr int kPolyPairsOf = kVariant == 0 ? 2 : 1;
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
  CUtensorMap tm_k;  // (128, Nk, B*Hkv)       box (64, 32, 1)
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

// Debug timeline (kFlagTimeline): CTA 0 (rank 0 of the first pair) stamps
// clock64() at fixed points of its first work item's first kTimelineBlocks
// key blocks.  Layout: u64 [role][block][event] at byte kTimelineOffset of
// the workspace; roles 0/1 = softmax tile 0/1 (warp 4t, lane 0), 2 = MMA
// threads, 3 = TMA thread.  Softmax events: 0 S low ready, 1 keys 0-63
// loaded, 2 row max / rescale decided, 3 P half handed over, 4 P full handed
// over.  MMA events of tile t's issuer at 4t + {0 iteration start, 1 "P
// half" seen, 2 "P full" seen, 3 second window issued}.  TMA events: 0/1 K
// wait/issue, 2/3 V wait/issue.
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

// Bounded mbarrier waits.  `site` identifies the wait in the status word:
// (rank << 16) | (warp << 8) | barrier slot.
struct Waiter {
  uint32_t abort_slot;       // shared u32, nonzero once any thread of the pair gave up
  uint32_t peer_abort_slot;  // the other CTA's abort flag (cluster address)
  uint64_t timeout_ns;
  uint32_t* ws;

  __device__ __forceinline__ void fail(uint32_t site) const {
    st_volatile_shared(abort_slot, 1u);
    st_cluster_u32(peer_abort_slot, 1u);
    if (atomicCAS(&ws[0], 0u, 1u /* B200FA_DEV_TIMEOUT */) == 0u) {
      ws[1] = site;
      ws[2] = blockIdx.x;
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
    while (!mbar_test_cluster(bar, parity)) {
      if (global_timer_ns() - t0 > limit_ns) return;
    }
  }
};

struct Smem {
  uint32_t base;  // shared-window address of the aligned base
  __device__ __forceinline__ uint32_t bar(int i) const { return base + kSmemBar + 8 * i; }
  __device__ __forceinline__ uint32_t q(int t) const { return base + kSmemQ + t * kQTileBytes; }
  __device__ __forceinline__ uint32_t kv(uint32_t s) const { return base + kSmemKV + s * kStageBytes; }
  __device__ __forceinline__ uint32_t tmem_slot() const { return base + kSmemMisc; }
  __device__ __forceinline__ uint32_t abort_slot() const { return base + kSmemMisc + 4; }
};

// Positions in the K/V ring count the CTA's key blocks over all its items:
// K of block g at 2g, V at 2g+1; slot = pos % kStages, use = pos / kStages.
__device__ __forceinline__ uint32_t ring_slot(uint32_t pos) { return pos % kStages; }
__device__ __forceinline__ uint32_t ring_parity(uint32_t pos) { return (pos / kStages) & 1u; }

// ------------------------------------------------------------------ roles
// Rank 0, one thread per tile: the pair's tensor-core work for tile t.
// Timeline events (role 2): issuer t uses events 4t .. 4t+3.
__device__ void mma_role(const FwdParams& p, const Smem& sm, uint32_t tmem_base, const Waiter& w, int t) {
  const uint32_t site = uint32_t(kMmaWarp + 2 * t) << 8;
  const int n = p.n_kv;
  const uint32_t q_lo = desc_lo(sm.q(t));
  const uint32_t ring_lo = desc_lo(sm.kv(0));   // + slot * (kStageBytes >> 4)
  const uint32_t tS = tmem_base + kTmemS + 128u * t;
  const uint32_t tO = tmem_base + kTmemO + 128u * t;
  uint32_t kv_base = 0;   // ring position of the current item's K_0
  uint32_t p_phase = 0;   // parity of "P half" / "P full" t
  bool ok = true;

  auto kv_ready = [&](uint32_t pos) -> bool {
    return w.wait(sm.bar(kBarKVFull + ring_slot(pos)), ring_parity(pos), site | kBarKVFull);
  };
  auto stage_lo = [&](uint32_t pos) -> uint32_t { return ring_lo + ring_slot(pos) * uint32_t(kStageBytes >> 4); };
  // One half (keys 0-63: h = 0, keys 64-127: h = 1) of S_t = Q_t K^T for
  // the block whose K sits at ring position `pos`, into S_t columns
  // [64h, 64h+64); each CTA supplies 32 keys of the half.
  auto issue_s_half = [&](uint32_t pos, int h) {
    mma_pair_ss_k128<uint32_t(kQHalfBytes >> 4), uint32_t(kKBoxBytes >> 4)>(
        tS + 64u * uint32_t(h), q_lo, stage_lo(pos) + uint32_t(h) * uint32_t(kKPartBytes >> 4), kDescHi, kIdescQK);
    mma_commit_pair_both(sm.bar((h == 0 ? kBarSLo : kBarSHi) + t));
  };

  for (int item = int(cluster_id_x()), it = 0; ok && item < p.num_items; item += int(num_clusters_x()), ++it) {
    const Timeline tl = make_timeline(p, it);
    const uint32_t ip = uint32_t(it) & 1u;
    if (!w.wait(sm.bar(kBarQFull + t), ip, site | (kBarQFull + t))) break;
    if (!kv_ready(kv_base)) break;
    tc_fence_after();
    issue_s_half(kv_base, 0);  // S_t(0)
    issue_s_half(kv_base, 1);
    for (int j = 0; j < n; ++j) {
      const uint32_t vpos = kv_base + 2u * uint32_t(j) + 1u;
      const bool more = j + 1 < n;
      tl.mark(2, j, 4 * t + 0);
      // Both stages first: after each PV half this thread touches no shared
      // memory before the S half that reuses its P columns.
      if (!kv_ready(vpos) || (more && !kv_ready(vpos + 1u))) { ok = false; break; }
      if (!w.wait(sm.bar(kBarPHalf + t), p_phase, site | (kBarPHalf + t))) { ok = false; break; }
      tl.mark(2, j, 4 * t + 1);
      tc_fence_after();
      // "P half": S_t(j) keys 0-63 are read (P sits in the upper columns),
      // so S_t(j+1) keys 0-63 go first and are ready early.
      if (more) issue_s_half(vpos + 1u, 0);
      mma_pair_ts_k64(tO, tS + kTmemPLo, stage_lo(vpos), kDescHi, kIdescPV, j == 0 ? 0u : 1u);
      if (!w.wait(sm.bar(kBarPFull + t), p_phase, site | (kBarPFull + t))) { ok = false; break; }
      p_phase ^= 1u;
      tl.mark(2, j, 4 * t + 2);
      tc_fence_after();
      mma_pair_ts_k64(tO, tS + kTmemPHi, stage_lo(vpos) + 4u * 128u, kDescHi, kIdescPV, 1u);
      if (more) issue_s_half(vpos + 1u, 1);  // keys 64-127, over both P halves: after both PV halves
      else mma_commit_pair_both(sm.bar(kBarOFinal + t));
      tl.mark(2, j, 4 * t + 3);
    }
    kv_base += 2u * uint32_t(n);
  }
  // All MMAs this thread issued must be complete before TMEM is freed.
  mma_commit_pair(sm.bar(kBarDrain + t));
  w.drain(sm.bar(kBarDrain + t), 0u, 100000000ull);
}

// Rank 1, one thread: replays the producer's sequence and, as each of this
// CTA's stages lands, arrives on the same barrier of rank 0 (whose MMAs read
// both CTAs' halves).
__device__ void forward_role(const FwdParams& p, const Smem& sm, const Waiter& w) {
  const uint32_t site = (1u << 16) | (uint32_t(kForwardWarp) << 8);
  const int n = p.n_kv;
  uint32_t pos = 0;
  auto forward = [&](int bar, uint32_t parity) -> bool {
    if (!w.wait(sm.bar(bar), parity, site | uint32_t(bar))) return false;
    mbar_arrive_cluster(map_shared(sm.bar(bar), 0));
    return true;
  };
  bool ok = true;
  for (int item = int(cluster_id_x()), it = 0; ok && item < p.num_items; item += int(num_clusters_x()), ++it) {
    const uint32_t ip = uint32_t(it) & 1u;
    if (!forward(kBarQFull + 0, ip)) break;
    for (int j = 0; j < n; ++j) {
      if (!forward(kBarKVFull + int(ring_slot(pos)), ring_parity(pos))) { ok = false; break; }
      ++pos;
      if (j == 0 && !forward(kBarQFull + 1, ip)) { ok = false; break; }
      if (!forward(kBarKVFull + int(ring_slot(pos)), ring_parity(pos))) { ok = false; break; }
      ++pos;
    }
  }
}

// Both ranks, one thread: this CTA's Q tiles and its halves of every K/V block.
__device__ void load_role(const FwdParams& p, const Smem& sm, const Waiter& w, uint32_t rank) {
  const uint32_t site = (rank << 16) | (uint32_t(kLoadWarp) << 8);
  const int n = p.n_kv;
  uint32_t kv_it = 0;
  uint32_t issued = 0;       // bit s: stage s has ever been loaded
  uint32_t last_par = 0;     // bit s: parity of stage s's last load
  uint32_t q_issued = 0, q_par = 0;
  bool ok = true;
  for (int item = int(cluster_id_x()), it = 0; ok && item < p.num_items; item += int(num_clusters_x()), ++it) {
    int bh, qb, cnt;
    plan_decode<int>(p.nqb, p.unit_begin, p.unit_end, item, bh, qb, cnt);
    const int b = bh / p.Hq;
    const int kvh = b * p.Hkv + (bh - b * p.Hq) / p.group;
    // Tile t of rank r is unit 2t+r; missing units of a short item repeat
    // the last one (computed, not stored).
    const int u0 = int(rank) < cnt ? int(rank) : cnt - 1;
    const int u1 = 2 + int(rank) < cnt ? 2 + int(rank) : cnt - 1;
    const int row0 = (qb + u0) * kBlockM;
    const int row1 = (qb + u1) * kBlockM;
    const uint32_t ip = uint32_t(it) & 1u;
    const Timeline tl = make_timeline(p, it);
    if (!w.wait(sm.bar(kBarQEmpty + 0), ip ^ 1u, site | (kBarQEmpty + 0))) break;
    mbar_arrive_expect_tx(sm.bar(kBarQFull + 0), kQTileBytes);
    tma_load_3d(sm.q(0), &p.tm_q, sm.bar(kBarQFull + 0), 0, row0, bh);
    tma_load_3d(sm.q(0) + kQHalfBytes, &p.tm_q, sm.bar(kBarQFull + 0), 64, row0, bh);
    q_issued |= 1u;
    q_par = (q_par & ~1u) | ip;
    for (int j = 0; j < n; ++j) {
#pragma unroll
      for (int which = 0; which < 2; ++which) {  // 0: K_j half, 1: V_j half
        const uint32_t s = ring_slot(kv_it);
        const uint32_t ph = ring_parity(kv_it);
        ++kv_it;
        tl.mark(3, j, 2 * which);
        if (!w.wait(sm.bar(kBarKVEmpty + s), ph ^ 1u, site | (kBarKVEmpty + s))) { ok = false; break; }
        tl.mark(3, j, 2 * which + 1);
        mbar_arrive_expect_tx(sm.bar(kBarKVFull + s), kStageBytes);
        if (which == 0) {  // keys [j*128 + 64h + 32r, +32) of each half h, all 128 head-dim columns
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int krow = j * kBlockN + h * (kBlockN / 2) + int(rank) * kKBoxRows;
            const uint32_t dst = sm.kv(s) + uint32_t(h * kKPartBytes);
            tma_load_3d(dst, &p.tm_k, sm.bar(kBarKVFull + s), 0, krow, kvh);
            tma_load_3d(dst + kKBoxBytes, &p.tm_k, sm.bar(kBarKVFull + s), 64, krow, kvh);
          }
        } else {           // keys [j*128, +128), head-dim columns [64r, +64)
          tma_load_3d(sm.kv(s), &p.tm_v, sm.bar(kBarKVFull + s), int(rank) * kPairDims, j * kBlockN, kvh);
        }
        issued |= 1u << s;
        last_par = (last_par & ~(1u << s)) | (ph << s);
        if (which == 0 && j == 0) {
          if (!w.wait(sm.bar(kBarQEmpty + 1), ip ^ 1u, site | (kBarQEmpty + 1))) { ok = false; break; }
          mbar_arrive_expect_tx(sm.bar(kBarQFull + 1), kQTileBytes);
          tma_load_3d(sm.q(1), &p.tm_q, sm.bar(kBarQFull + 1), 0, row1, bh);
          tma_load_3d(sm.q(1) + kQHalfBytes, &p.tm_q, sm.bar(kBarQFull + 1), 64, row1, bh);
          q_issued |= 2u;
          q_par = (q_par & ~2u) | (ip << 1);
        }
      }
      if (!ok) break;
    }
  }
  // Copies still in flight must land before the CTA exits (only possible on
  // the abort path; on the normal path rank 0's MMAs consumed every stage).
  if (!ok || ld_volatile_shared(sm.abort_slot()) != 0u) {
    for (int s = 0; s < kStages; ++s)
      if (issued & (1u << s)) w.drain(sm.bar(kBarKVFull + s), (last_par >> s) & 1u, 50000000ull);
    for (int t = 0; t < 2; ++t)
      if (q_issued & (1u << t)) w.drain(sm.bar(kBarQFull + t), (q_par >> t) & 1u, 50000000ull);
  }
}

// Exponentials of 16*kGroups keys (8 pairs per group) of one row:
// x = s * scale*log2(e) - m with packed FP32 FMAs; of every 8 pairs the last
// kPoly go through the FMA-pipe polynomial (exp2_poly2) and the rest through
// MUFU (FP32 ex2).  Writes 8*kGroups packed FP16 pairs of P and adds the
// row sum: FP32 variant, the FP32 exponentials into packed FP32 sums (four
// chains, folded into acc0/acc1); FP16 variant, the FP16 P itself into
// packed FP16 sums (four chains; at most 16*kGroups <= 64 terms of <= 2^8,
// far inside FP16 range), carried over to FP32 once per call (hsum).
template <int kVariant, int kPoly, int kGroups>
__device__ __forceinline__ void exp_keys(const uint32_t* r, uint64_t sl2x2, uint64_t nmx2, uint32_t* pk,
                                         uint64_t& acc0, uint64_t& acc1, float& hsum) {
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
      else hc[pp & 3] = (g == 0 && pp < 4) ? pk[i] : hadd2(hc[pp & 3], pk[i]);
    }
  }
  if constexpr (kVariant == 0) hsum += h2_sum_f32(hadd2(hadd2(hc[0], hc[1]), hadd2(hc[2], hc[3])));
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

// Keys at or beyond `valid` (the last block's key count) get score -inf.
__device__ __forceinline__ void mask_keys64(uint32_t* r, int first_key, int valid) {
#pragma unroll
  for (int i = 0; i < 64; ++i)
    if (first_key + i >= valid) r[i] = __float_as_uint(-INFINITY);
}

// Scores of keys [first, first+64) of this thread's row from TMEM.
__device__ __forceinline__ void load_keys64(uint32_t tS, int first, uint32_t* r, bool tail, int valid) {
  tmem_ld32(tS + uint32_t(first), r);
  tmem_ld32(tS + uint32_t(first) + 32u, r + 32);
  tmem_wait_ld();
  if (tail) mask_keys64(r, first, valid);
}

// Softmax of one query tile per warpgroup (warps 0-3: tile 0, 4-7: tile 1),
// one thread per query row (its TMEM lane), in both CTAs.
// kCapture: the debug-capture instantiation (separate kernels, so the
// production ones carry no capture code).
template <int kVariant, bool kCapture>  // kVariant 0 = FP16 softmax, 1 = FP32 softmax
__device__ void softmax_role(const FwdParams& p, const Smem& sm, uint32_t tmem_base, const Waiter& w,
                             uint32_t warp, uint32_t lane, uint32_t rank) {
  const int t = int(warp >> 2);   // tile = warpgroup
  const int wq = int(warp & 3);   // TMEM lane quarter of this warp
  const int row = wq * 32 + int(lane);
  const uint32_t lane_off = uint32_t(wq * 32) << 16;
  const uint32_t tS = tmem_base + lane_off + kTmemS + uint32_t(t) * 128;
  const uint32_t tO = tmem_base + lane_off + kTmemO + uint32_t(t) * 128;
  const uint32_t sQ = sm.q(t);
  const uint32_t site = (rank << 16) | (warp << 8);
  const float sl2 = p.scale_log2;
  const uint64_t sl2x2 = f2_pack(sl2, sl2);
  const int n = p.n_kv;
  const bool withhold = (p.flags & kFlagTestWithholdP) != 0 && t == 1;
  // P half / P full live in rank 0; each warp arrives once (lane 0), after
  // its TMEM writes completed (tcgen05.wait::st), so rank 1's remote
  // arrival can be relaxed.
  const uint32_t p_half = rank == 0 ? sm.bar(kBarPHalf + t) : map_shared(sm.bar(kBarPHalf + t), 0);
  const uint32_t p_full = rank == 0 ? sm.bar(kBarPFull + t) : map_shared(sm.bar(kBarPFull + t), 0);
  auto arrive_rank0 = [&](uint32_t bar) {
    __syncwarp();
    if (lane == 0) {
      if (rank == 0) mbar_arrive(bar);
      else mbar_arrive_cluster_relaxed(bar);
    }
  };
  // One thread per tile returns this tile's use of the K/V ring slots to
  // the CTA's producer (a slot takes one arrival per tile): K of block g
  // once "S high t" g completed, V of block g once "S high t" g+1 (or "O
  // final t") completed.
  const bool releaser = wq == 0 && lane == 0;
  uint32_t g = 0;        // key blocks of this CTA so far (ring positions 2g, 2g+1)
  uint32_t s_phase = 0;  // parity of "S low t" / "S high t"
  bool ok = true;

  for (int item = int(cluster_id_x()), it = 0; ok && item < p.num_items; item += int(num_clusters_x()), ++it) {
    float m_ref = -INFINITY;  // reference maximum, log2 domain
    float l = 0.f;
    const Timeline tl = (wq == 0 && lane == 0) ? make_timeline(p, it) : Timeline{nullptr};
    // Debug capture: cap_on is warp-uniform (this tile holds a unit of the
    // item), cap_row per thread (its query row exists).  Record (b*Hq+hq,
    // block j, row) sits at index (bh*n + j)*nq + row of each scalar plane
    // (stride heads*n*nq) and, times 128, in the O plane after them.
    bool cap_on = false, cap_row = false;
    size_t cap_idx = 0;
    if constexpr (kCapture) {
      int bh, qb, cnt;
      plan_decode<int>(p.nqb, p.unit_begin, p.unit_end, item, bh, qb, cnt);
      const int u = 2 * t + int(rank);
      const int qrow = (qb + u) * kBlockM + row;
      cap_on = u < cnt;
      cap_row = cap_on && qrow < p.nq;
      cap_idx = (size_t(bh) * size_t(n)) * size_t(p.nq) + size_t(qrow);
    }
    const size_t cap_plane = size_t(p.heads) * size_t(n) * size_t(p.nq);
    // O after PV_t(jb) (unnormalised FP32, relative to that block's m):
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

    for (int j = 0; j < n; ++j, ++g) {
      // Keys 0-63 ("S low" j; it also means PV_t(j-1) keys 0-63 are done):
      // load, exponentiate speculatively against the current reference
      // (after the first block), and reduce their maximum.
      if (!w.wait(sm.bar(kBarSLo + t), s_phase, site | (kBarSLo + t))) { ok = false; break; }
      tl.mark(t, j, 0);
      tc_fence_after();
      const bool tail = (j == n - 1 && p.nk_tail < kBlockN);
      uint32_t pk[kBlockN / 2];
      uint64_t acc0 = 0ull, acc1 = 0ull;  // packed FP32 partial row sums
      float hsum = 0.f;                   // FP16 variant: sums of FP16 group sums
      float mx;
      {
        uint32_t r[64];
        load_keys64(tS, 0, r, tail, p.nk_tail);
        tl.mark(t, j, 1);
        if (j > 0) exp_keys<kVariant, kPolyPairsOf<kVariant>, 4>(r, sl2x2, f2_pack(-m_ref, -m_ref), pk, acc0, acc1, hsum);
        mx = row_max64(r);
      }
      // Keys 64-127 ("S high" j: S_t(j) and PV_t(j-1) complete): load and
      // reduce (their exponentials follow the check).
      if (!w.wait(sm.bar(kBarSHi + t), s_phase, site | (kBarSHi + t))) { ok = false; break; }
      s_phase ^= 1u;
      if (releaser) {
        mbar_arrive(sm.bar(kBarKVEmpty + ring_slot(2u * g)));                  // S_t(j) read K_j
        if (j > 0) mbar_arrive(sm.bar(kBarKVEmpty + ring_slot(2u * g - 1u)));  // PV_t(j-1) read V_(j-1)
      }
      tc_fence_after();
      if constexpr (kCapture) {
        if (cap_on && j > 0) capture_o(j - 1);
      }
      uint32_t r1[64];
      load_keys64(tS, 64, r1, tail, p.nk_tail);
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
      if (__any_sync(0xffffffffu, moved)) {
        // Lazy correction of the running output before any of this block's
        // P is handed over (PV_t(j-1) is complete: "S high" j covers it;
        // the P stores' wait below also covers these stores).  Then keys
        // 0-63 again from S, which is intact until P is written.
        if (j > 0) {
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
        uint32_t r[64];
        load_keys64(tS, 0, r, tail, p.nk_tail);
        if (moved) {
          acc0 = 0ull;
          acc1 = 0ull;
          hsum = 0.f;
          exp_keys<kVariant, kPolyPairsOf<kVariant>, 4>(r, sl2x2, f2_pack(-m_ref, -m_ref), pk, acc0, acc1, hsum);
        }
      }
      tmem_st32(tS + kTmemPLo, pk);
      tmem_wait_st();
      tc_fence_before();
      arrive_rank0(p_half);
      tl.mark(t, j, 3);
      exp_keys<kVariant, kPolyPairsOf<kVariant>, 4>(r1, sl2x2, f2_pack(-m_ref, -m_ref), pk + 32, acc0, acc1, hsum);
      tmem_st32(tS + kTmemPHi, pk + 32);
      tmem_wait_st();
      tc_fence_before();
      if (!(withhold && it == 0 && j == 0)) arrive_rank0(p_full);
      tl.mark(t, j, 4);
      float a0, b0, a1, b1;
      f2_unpack(acc0, a0, b0);
      f2_unpack(acc1, a1, b1);
      const float z = ((a0 + b0) + (a1 + b1)) + hsum;
      l += z;
      if constexpr (kCapture) {
        if (cap_row) {
          float* rec = p.capture + cap_idx + size_t(j) * size_t(p.nq);
          rec[0] = m_ref;
          rec[cap_plane] = l;
          rec[2 * cap_plane] = j == 0 ? 0.f : alpha;
          rec[3 * cap_plane] = z;
        }
      }
    }
    if (!ok) break;

    // ---- epilogue: O / l -> FP16 -> swizzled smem (this tile's Q buffer) -> TMA store
    if (!w.wait(sm.bar(kBarOFinal + t), uint32_t(it) & 1u, site | (kBarOFinal + t))) { ok = false; break; }
    if (releaser) mbar_arrive(sm.bar(kBarKVEmpty + ring_slot(2u * g - 1u)));  // V of the item's last block
    tc_fence_after();
    if constexpr (kCapture) {
      if (cap_on) capture_o(n - 1);
    }
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
        const uint32_t addr = sQ + uint32_t(gu >> 3) * kQHalfBytes + uint32_t(row) * 128 +
                              (uint32_t((gu & 7) ^ (row & 7)) << 4);
        st_shared_v4(addr, h0, h1, h2, h3);
      }
    }
    tc_fence_before();
    fence_proxy_async_smem();
    mbar_arrive(sm.bar(kBarOStaged + t));
    if (wq == 0 && lane == 0) {
      int bh, qb, cnt;
      plan_decode<int>(p.nqb, p.unit_begin, p.unit_end, item, bh, qb, cnt);
      if (!w.wait(sm.bar(kBarOStaged + t), uint32_t(it) & 1u, site | (kBarOStaged + t))) {
        ok = false;
      } else {
        const int u = 2 * t + int(rank);
        if (u < cnt) {
          const int orow = (qb + u) * kBlockM;
          tma_store_3d(&p.tm_o, sQ, 0, orow, bh);
          tma_store_3d(&p.tm_o, sQ + kQHalfBytes, 64, orow, bh);
          bulk_commit_group();
          bulk_wait_group_read0();
        }
        mbar_arrive(sm.bar(kBarQEmpty + t));
      }
    }
  }
  if (wq == 0 && lane == 0) bulk_wait_group0();
}

template <int kVariant, bool kCapture>
__device__ __forceinline__ void attention_fwd_body(const FwdParams& p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  Smem sm{(raw + 1023u) & ~1023u};
  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_rank();
  const uint64_t t_start = global_timer_ns();

  if (threadIdx.x == 0) {
    const uint32_t fed = rank == 0 ? 2u : 1u;  // rank 0's full barriers also count rank 1's forward
    for (int t = 0; t < 2; ++t) {
      mbar_init(sm.bar(kBarQFull + t), fed);
      mbar_init(sm.bar(kBarQEmpty + t), 1);
      mbar_init(sm.bar(kBarPHalf + t), kTileWarps);
      mbar_init(sm.bar(kBarPFull + t), kTileWarps);
      mbar_init(sm.bar(kBarOStaged + t), 128);
      mbar_init(sm.bar(kBarSLo + t), 1);
      mbar_init(sm.bar(kBarSHi + t), 1);
      mbar_init(sm.bar(kBarOFinal + t), 1);
      mbar_init(sm.bar(kBarDrain + t), 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(sm.bar(kBarKVFull + s), fed);
      mbar_init(sm.bar(kBarKVEmpty + s), 2);  // one release per tile
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
    tmem_alloc_pair(sm.tmem_slot(), kTmemCols);
    tmem_relinquish_pair();
  }
  // Barriers of both CTAs initialised and TMEM allocated before any
  // cross-CTA arrival or pair MMA.
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = ld_volatile_shared(sm.tmem_slot());
  const Waiter w{sm.abort_slot(), map_shared(sm.abort_slot(), rank ^ 1u), p.timeout_ns, p.ws};

  if (warp < 8) {
    regs_increase<kSoftmaxRegs>();
    softmax_role<kVariant, kCapture>(p, sm, tmem_base, w, warp, lane, rank);
  } else {
    regs_decrease<kControlRegs>();
    if (lane == 0) {
      if (rank == 0 && (warp == kMmaWarp || warp == kMmaWarp + 2)) mma_role(p, sm, tmem_base, w, int(warp - kMmaWarp) / 2);
      else if (warp == kLoadWarp) load_role(p, sm, w, rank);
      else if (rank == 1 && warp == kForwardWarp) forward_role(p, sm, w);
    }
  }
  __syncwarp();
  // Rank 0's MMAs read and write both CTAs' memories: neither CTA frees
  // TMEM or leaves before the pair is done.
  tc_fence_before();
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if ((p.flags & kFlagTrace) && threadIdx.x == kLoadWarp * 32 && blockIdx.x < 1024) {
    uint32_t* rec = p.ws + (256 + 32 * blockIdx.x) / 4;
    int items = 0;
    for (int item = int(cluster_id_x()); item < p.num_items; item += int(num_clusters_x())) ++items;
    const uint64_t t_end = global_timer_ns();
    rec[0] = sm_id();
    rec[1] = uint32_t(items);
    rec[2] = uint32_t(t_start);
    rec[3] = uint32_t(t_start >> 32);
    rec[4] = uint32_t(t_end);
    rec[5] = uint32_t(t_end >> 32);
    rec[6] = rank;
    rec[7] = 0u;
  }
}

}  // namespace b200fa
