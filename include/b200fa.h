/*
 * b200fa.h -- C ABI of libb200fa.so, the sm_100a flash-attention forward.
 *
 * One operator: non-causal grouped-query attention forward,
 *     O[b,h] = softmax(Q[b,h] K[b,kv(h)]^T * scale) V[b,kv(h)],
 *     kv(h) = h / (Hq / Hkv),
 * with FP16 Q [B,Hq,Nq,128], K and V [B,Hkv,Nk,128] and FP16 normalized
 * O [B,Hq,Nq,128], all contiguous (BHND, "BNSD" in torch_npu terms).
 *
 * This library replaces the native call pair of the reference's CCE
 * backends,
 *   aclnn<Op>GetWorkspaceSize(q, k, v, q_block, k_block, q_l1, groups,
 *                             capture, phase, [gray], sp, partial, trace,
 *                             stats, running, output, &ws_size, &executor)
 *   aclnn<Op>(workspace, ws_size, executor, stream)
 * bound in backends/cce_fa_nqkq_nz_resident_v13_q768_pool_i4_p128/binding.py:20-26
 * and called at binding.py:72-80 (the FP32 twin,
 * backends/cce_fa_nk_nz_vector_fp32_v5_sumpack/binding.py, has the same
 * shape).  The ACLNN executor and its tiling (op_host/*.cpp:53-89) collapse
 * into the plain-pointer call b200fa_fwd below; the host-side shape checks of
 * binding.py:87-98 and op_host/*.cpp:8-19 become the negative return codes.
 *
 * Conventions
 *   - All tensor pointers are CUDA device pointers owned by the caller; the
 *     library allocates no device memory and keeps no per-call state.
 *   - Calls are asynchronous on the caller's stream (cudaStream_t passed as
 *     void*, NULL = legacy default stream); nothing synchronizes implicitly
 *     except b200fa_read_status.
 *   - Return value 0 = success, negative = argument validation error (no
 *     CUDA call was made), positive = CUDA runtime error code from a launch
 *     or attribute call.  b200fa_last_error_string() describes the last
 *     failure on the calling thread.
 *   - Device-side failures (a bounded wait that ran out) do not abort the
 *     kernel's caller: the kernel records a status word in the workspace
 *     and returns; b200fa_read_status() reads it.
 */
#ifndef B200FA_H_
#define B200FA_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Variant selector: softmax arithmetic of the two shipped kernels.
 * B200FA_VARIANT_FP16 mirrors the reference CCE FP16 kernel
 *   (backends/cce_fa_nqkq_nz_resident_v13_q768_pool_i4_p128): row sums in
 *   FP16 partial sums of the FP16 P (FP32 exponentials).
 * B200FA_VARIANT_FP32 mirrors the CCE FP32 kernel
 *   (backends/cce_fa_nk_nz_vector_fp32_v5_sumpack): FP32 softmax throughout.
 * Both keep P in FP16 for the tensor-core PV product and accumulate O in
 * FP32 in tensor memory. */
#define B200FA_VARIANT_FP16 0
#define B200FA_VARIANT_FP32 1

/* Status / error codes. */
#define B200FA_OK                 0
#define B200FA_ERR_NULL          -1   /* a required pointer is NULL            */
#define B200FA_ERR_HEAD_DIM      -2   /* D != 128                              */
#define B200FA_ERR_SHAPE         -3   /* B, Hq, Hkv, Nq or Nk <= 0             */
#define B200FA_ERR_GROUPING      -4   /* Hq % Hkv != 0                         */
#define B200FA_ERR_TOO_LARGE     -5   /* Nq, Nk or unit count >= 2^31          */
#define B200FA_ERR_UNIT_RANGE    -6   /* unit range outside [0, num_units]     */
#define B200FA_ERR_ALIGNMENT     -7   /* a tensor pointer is not 16-B aligned  */
#define B200FA_ERR_WORKSPACE     -8   /* workspace NULL, misaligned or small   */
#define B200FA_ERR_VARIANT       -9   /* unknown variant                       */
#define B200FA_ERR_SCALE        -10   /* scale not finite or not positive      */
#define B200FA_ERR_OPTIONS      -11   /* malformed b200fa_options              */
#define B200FA_ERR_NO_DRIVER    -12   /* cuTensorMapEncodeTiled unavailable    */
#define B200FA_ERR_TENSOR_MAP   -13   /* cuTensorMapEncodeTiled rejected a map */

/* Device status word values (b200fa_read_status, status[0]). */
#define B200FA_DEV_OK             0
#define B200FA_DEV_TIMEOUT        1   /* a bounded mbarrier wait ran out       */
/* Checking build only (libb200fa_debug.so, compiled with B200FA_DEBUG): */
#define B200FA_DEV_BOUNDS         2   /* a coordinate, index or layout check failed;
                                         site low byte = 0x80 + check number    */
#define B200FA_DEV_PHASE          3   /* the roles' key-block counts disagreed at exit */

/* Option flags (b200fa_options.flags). */
#define B200FA_FLAG_TRACE          1u /* write one trace record per CTA        */
/* Test-only: softmax group 1 (the odd key blocks, in both CTAs of every
 * pair) withholds its first P-ready arrival, so the PV issuer's bounded
 * wait runs out and the kernel reports B200FA_DEV_TIMEOUT.  Used by the
 * failure-detection test only. */
#define B200FA_FLAG_TEST_WITHHOLD_P 2u
/* Debug, checking build only (libb200fa_debug.so; the product build ignores
 * the flag): both CTAs of the first pair record SM-clock timestamps of their
 * softmax, MMA-issuer / forwarder and TMA threads for the first
 * B200FA_TIMELINE_BLOCKS key blocks of their first work item into the
 * timeline area of the workspace (pipeline analysis). */
#define B200FA_FLAG_TIMELINE       4u
/* Debug capture (the counterpart of the reference's `capture` attribute,
 * binding.py:39-41, vector_output.h:94-106): per key block and query row the
 * kernel writes its online-softmax state into b200fa_options.capture, FP32,
 * laid out [plane][b*Hq + hq][key block][query row] with planes
 *   0  m      reference maximum after the block (log2 domain: scores times
 *             scale*log2(e)); it moves only when a block maximum exceeds it
 *             by more than 8 (lazy rescaling)
 *   1  l      running row sum after the block, relative to m
 *   2  alpha  factor applied to l and O at this block (2^(m_old - m_new);
 *             1 when m did not move, 0 at the first block)
 *   3  z      the block's own row sum, relative to m
 * followed by the O plane, [b*Hq + hq][key block][query row][128]:
 *   O after the block's P V product (unnormalised, relative to m); the
 *   block's own partial product is O_j - alpha_j * O_(j-1).
 * The reference's capture holds the same (m, l, alpha, z, O) per packet.
 * Key blocks are B200FA_BLOCK_KEYS keys wide.  Rows of the unit range only;
 * other entries are left untouched.  The buffer must be 16-byte aligned;
 * size: b200fa_capture_bytes() = 528 * B * Hq * ceil(Nk / 128) * Nq.  The
 * capture serialises each block's softmax with its P V product: a debug
 * mode, not a fast path. */
#define B200FA_FLAG_CAPTURE        8u
/* Test-only, checking build only: the producer offsets its first Q tile's
 * row coordinate past the end of the problem; the bounds check catches it
 * before the copy is issued and the kernel reports B200FA_DEV_BOUNDS.  The
 * product build ignores the flag (it has no checks and never offsets). */
#define B200FA_FLAG_TEST_BOUNDS   16u
/* Causal mask (top-left aligned, as torch's is_causal): query row i attends
 * keys 0..i only.  Key blocks past the diagonal of a work item's last query
 * block are skipped; the block that crosses a row's diagonal is masked.
 * Runs separate kernels (b200_fa_fp{16,32}_causal_kernel); not combined
 * with B200FA_FLAG_CAPTURE (B200FA_ERR_OPTIONS). */
#define B200FA_FLAG_CAUSAL        32u
#define B200FA_BLOCK_KEYS        128

typedef struct b200fa_options {
    uint32_t struct_size;   /* sizeof(b200fa_options); 16 (no capture fields)
                               is accepted too                               */
    uint32_t flags;         /* B200FA_FLAG_*                                  */
    uint32_t timeout_us;    /* bound of every device-side wait; 0 = 2 s       */
    int32_t  max_ctas;      /* cap on the persistent grid (CTAs; rounded down
                               to whole pairs, at least one pair); <= 0 = one
                               pair per TPC                                  */
    float*   capture;       /* B200FA_FLAG_CAPTURE: device buffer             */
    uint64_t capture_bytes; /* its size, >= b200fa_capture_bytes(...)        */
} b200fa_options;

/* Workspace layout (bytes, 256-B aligned, zeroed once by the owner):
 *   [0, 256)       status header: u32 status, u32 site, u32 cta, u32 spare...
 *                  site = (pair rank << 16) | (warp << 8) | barrier slot of
 *                  the first wait that ran out
 *   [256, 256 + 32 * B200FA_MAX_CTAS)
 *                  trace records, one per CTA (B200FA_FLAG_TRACE):
 *                  {u32 smid, u32 items, u64 t_start_ns, u64 t_end_ns,
 *                   u32 pair rank, u32 0}; both CTAs of a pair count the
 *                  pair's items
 *   [B200FA_WS_TIMELINE_OFFSET, + B200FA_WS_TIMELINE_BYTES)
 *                  timeline (B200FA_FLAG_TIMELINE): u64 clock64 stamps,
 *                  [pair rank 0..1][role 0..B200FA_TIMELINE_ROLES-1]
 *                  [block 0..B200FA_TIMELINE_BLOCKS-1][event 0..7], roles =
 *                  softmax warps 0-7, MMA issuers (rank 0) / forwarder
 *                  (rank 1), TMA.
 * The status is sticky: it stays set until b200fa_reset_status. */
#define B200FA_WS_HEADER_BYTES 256u
#define B200FA_WS_TRACE_BYTES   32u
#define B200FA_MAX_CTAS       1024
#define B200FA_TIMELINE_BLOCKS  48u
#define B200FA_TIMELINE_ROLES   10u
#define B200FA_WS_TIMELINE_OFFSET (B200FA_WS_HEADER_BYTES + B200FA_WS_TRACE_BYTES * B200FA_MAX_CTAS)
#define B200FA_WS_TIMELINE_BYTES  (2u * B200FA_TIMELINE_ROLES * B200FA_TIMELINE_BLOCKS * 8u * 8u)

/* Number of work units: (b, hq, 128-row query block) triples, linearised as
 * ((b * Hq) + hq) * ceil(Nq / 128) + qb -- the order of the reference's
 * task split, cce_task.h:28-35 / panel_kernel.h:264-274.  Returns a negative
 * validation code for non-positive sizes. */
int64_t b200fa_num_units(int64_t B, int64_t Hq, int64_t Nq);

/* Contiguous near-equal split of [0, total) into `parts` ranges, remainder to
 * the first parts -- the semantics of cce::PartitionContiguous
 * (cce_task.h:28-35).  Writes part `index`'s [begin, end).  0 or
 * B200FA_ERR_UNIT_RANGE. */
int b200fa_partition(int64_t total, int32_t parts, int32_t index,
                     int64_t* begin, int64_t* end);

/* Bytes of workspace b200fa_fwd needs (header + trace area for the maximum
 * grid).  Replaces aclnn<Op>GetWorkspaceSize (binding.py:72-77); the value
 * does not depend on the shape beyond validation.  Negative on invalid
 * arguments. */
int64_t b200fa_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq,
                              int64_t Nk, int64_t D, int32_t variant);

/* Attention forward over work units [unit_begin, unit_end) (the whole
 * problem is [0, b200fa_num_units(B, Hq, Nq))).  Rows of O outside the range
 * are not written.  Replaces aclnn<Op> (binding.py:72-80) and the tiling
 * kernel launch (op_host/*.cpp:53-89, panel_kernel.h:216-343). */
int b200fa_fwd(const void* q, const void* k, const void* v, void* o,
               int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq, int64_t Nk,
               int64_t D, float scale, int32_t variant,
               int64_t unit_begin, int64_t unit_end,
               void* workspace, uint64_t ws_bytes, void* stream);

/* b200fa_fwd with options (trace records, wait bound, grid cap, test
 * flags).  opts may be NULL. */
int b200fa_fwd_ex(const void* q, const void* k, const void* v, void* o,
                  int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq, int64_t Nk,
                  int64_t D, float scale, int32_t variant,
                  int64_t unit_begin, int64_t unit_end,
                  void* workspace, uint64_t ws_bytes, void* stream,
                  const b200fa_options* opts);

/* Synchronizes `stream`, then copies the 4-word status header of `workspace`
 * into status[0..3] = {status, site, cta, spare}.  Returns 0 or a CUDA error. */
int b200fa_read_status(const void* workspace, void* stream, uint32_t* status);

/* Clears the status header (async on `stream`). */
int b200fa_reset_status(void* workspace, void* stream);

/* Kernel symbol of a variant ("b200_fa_fp16_kernel" / "b200_fa_fp32_kernel"),
 * the names the harness profiler matches backends by; NULL for a bad id. */
const char* b200fa_kernel_name(int32_t variant);

/* Host-side work-item plan (no GPU): item `index` of the range
 * [unit_begin, unit_end) as {bh, first q-block, count (1..2)}: up to two
 * consecutive query blocks of one head, one per CTA of a pair.  Returns
 * the number of items, or a negative code. */
int64_t b200fa_plan_item(int64_t B, int64_t Hq, int64_t Nq,
                         int64_t unit_begin, int64_t unit_end, int64_t index,
                         int64_t* bh, int64_t* qblock, int64_t* count);

/* Bytes of the B200FA_FLAG_CAPTURE buffer:
 * 528 * B * Hq * ceil(Nk / B200FA_BLOCK_KEYS) * Nq (four scalar FP32 planes
 * and the 128-float O plane).  Negative on invalid sizes. */
int64_t b200fa_capture_bytes(int64_t B, int64_t Hq, int64_t Nq, int64_t Nk);

/* Description of the last error on the calling thread ("" if none). */
const char* b200fa_last_error_string(void);

/* Library version string. */
const char* b200fa_version(void);

/* Test hook, no counterpart in the reference: evaluates the softmax's two
 * exponential forms elementwise on n device floats, asynchronously on
 * `stream` -- poly[i] = the FMA-pipe 2^x the kernels use for part of every
 * row (Cody-Waite split, degree-3 minimax polynomial, input clamped at -120),
 * mufu[i] = the MUFU ex2.approx.ftz form they use for the rest.  Lets a test
 * check the compiled device function against exp2 over the softmax's input
 * range.  0, B200FA_ERR_NULL, B200FA_ERR_SHAPE (n < 0 or >= 2^31) or a CUDA
 * error code. */
int b200fa_test_exp2(const float* x, float* poly, float* mufu, int64_t n, void* stream);

/* Allocation-free forward.  This entry point has no counterpart in the
 * reference; it exists for callers that cannot hand the library a
 * workspace: a C or FFI host with no device allocator of its own, a runtime
 * that has reserved the whole device pool for itself and forbids side
 * allocations, or a latency-critical path that must not call cudaMalloc
 * (which can synchronize the device).  Same computation and arguments as
 * b200fa_fwd_ex minus the workspace: the status header and trace records
 * live in a static device array of B200FA_NOALLOC_SCRATCH_BYTES bytes
 * (256-byte header + trace records for at most B200FA_NOALLOC_TRACE_CTAS
 * CTAs), one copy on every device that loads the library, held until the
 * process exits.  Nothing is allocated: no cudaMalloc, cudaFree or
 * allocating library routine is called.
 *   - The first call on a device resolves that device's copy of the array
 *     (cudaGetSymbolAddress) and sets the kernel attributes; make that first
 *     call before any stream capture.
 *   - Each call clears the status header on `stream` before its launch.
 *     All calls share the array: calls that overlap on the GPU (e.g. on
 *     different streams) race on the status header and trace records.
 *   - A call whose scratch need exceeds the array -- tracing
 *     (B200FA_FLAG_TRACE) with a persistent grid of more than
 *     B200FA_NOALLOC_TRACE_CTAS CTAs -- is rejected with
 *     B200FA_ERR_WORKSPACE before anything is launched; cap the grid with
 *     opts->max_ctas or trace less.  B200FA_FLAG_TIMELINE is not supported
 *     here (its area alone exceeds the array) and is rejected the same way.
 *   - A call with an empty unit range launches nothing but still clears the
 *     status header, so a status read afterwards describes this call.
 *   - scratch_out (may be NULL) receives the device address of this
 *     device's scratch, for b200fa_read_status / b200fa_reset_status. */
#define B200FA_NOALLOC_TRACE_CTAS 128u
#define B200FA_NOALLOC_SCRATCH_BYTES \
    (B200FA_WS_HEADER_BYTES + B200FA_WS_TRACE_BYTES * B200FA_NOALLOC_TRACE_CTAS)
int b200fa_fwd_noalloc(const void* q, const void* k, const void* v, void* o,
                       int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq, int64_t Nk,
                       int64_t D, float scale, int32_t variant,
                       int64_t unit_begin, int64_t unit_end,
                       void* stream, const b200fa_options* opts, void** scratch_out);

#ifdef __cplusplus
}
#endif

#endif /* B200FA_H_ */
