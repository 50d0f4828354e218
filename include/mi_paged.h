/*
 * mi_paged.h -- C ABI of the B200-native paged-KV hot path of minimal-inference.
 *
 * One shared library (libmi_paged.so, sm_100a) exports these entry points.
 * Every argument is a plain pointer or size: device pointers point into
 * caller-owned CUDA memory, `stream` is a cudaStream_t (NULL = legacy default
 * stream). Nothing here allocates device memory, synchronises the stream or
 * reads device memory from the host, so every call can be captured into a
 * CUDA graph.
 *
 * Two error channels:
 *   - the return value (MI_OK or an MI_ERR_* code) reports argument and
 *     launch errors found on the host; mi_last_error() gives the message;
 *   - kernels never trap: problems found on the device (page pool exhausted,
 *     a page id outside the pool, ...) are OR-ed as MI_STATUS_* bits into an
 *     optional caller-owned int32 in device memory (`status`), which the
 *     caller reads whenever it next synchronises.
 *
 * Page pool layout (one tensor per layer), as the reference's PagedKVCache
 * (scheduler.py:194-202) and FlashInfer's NHD layout define it:
 *     kv_data[num_pages][2][page_size][num_kv_heads][head_dim], K at [.][0].
 * Page tables are CSR: kv_indptr[batch+1], kv_indices[kv_indptr[batch]],
 * kv_last_page_len[batch]; a request with n > 0 pages holds
 * (n-1)*page_size + last_page_len tokens, one with 0 pages holds none.
 */
#ifndef MI_PAGED_H
#define MI_PAGED_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *mi_stream_t;

/* element type of q / k / v / out / the page pool */
enum { MI_DTYPE_F32 = 0, MI_DTYPE_F16 = 1, MI_DTYPE_BF16 = 2 };

/* host-side return codes */
enum {
  MI_OK = 0,
  MI_ERR_INVALID = 1,     /* bad argument (shape, alignment, null pointer) */
  MI_ERR_UNSUPPORTED = 2, /* valid but not supported by this build */
  MI_ERR_WORKSPACE = 3,   /* workspace too small */
  MI_ERR_CUDA = 4         /* a CUDA runtime call or launch failed */
};

/* device-side status bits (OR-ed into *status) */
enum {
  MI_STATUS_OUT_OF_PAGES = 1,    /* allocation larger than the free list: nothing popped */
  MI_STATUS_BAD_PAGE = 2,        /* a page id outside [0, num_pages): access skipped */
  MI_STATUS_BAD_POSITION = 4,    /* token position outside its pages / RoPE table: skipped */
  MI_STATUS_BAD_BATCH_INDEX = 8, /* batch index outside [0, batch_size): skipped */
  MI_STATUS_POOL_OVERFLOW = 16,  /* release would overfill the free list (double free) */
  MI_STATUS_SLOT_FULL = 32,      /* a slot's page table row is full: nothing popped */
  MI_STATUS_TIMEOUT = 64         /* a bounded device-side wait gave up: results invalid */
};

/* Message for the last non-OK return on this thread ("" if none). */
const char *mi_last_error(void);
/* Library ABI version (major*100 + minor). */
int mi_version(void);

/* ---------------------------------------------------------------------------
 * (1) KV append with fused RoPE
 *
 * Replaces flashinfer.page.append_paged_kv_cache as model.py:207-216 calls
 * it (flashinfer page.py:280-290; addressing page.cuh:259-283): token i of
 * request b = batch_indices[i] at position p = positions[i] goes to page
 * kv_indices[kv_indptr[b] + p/page_size], slot p%page_size; its K row to
 * kv_data[page][0][slot], its V row to kv_data[page][1][slot]. Rows are
 * [num_kv_heads][head_dim] with the given token/head strides (elements).
 *
 * When rope_cos/rope_sin are given ([rope_max_pos][head_dim] tables in
 * `dtype`), K is rotated before it is stored, with the rounding of
 * apply_rotary_emb (model.py:92-107, called at :170): bit-identical to the
 * reference's pages. RoPE positions are rope_positions[i] (or positions[i]
 * when NULL). When q_in is also given, the same launch writes the rotated
 * query rows ([nnz][num_qo_heads][head_dim]) to q_out (model.py:169);
 * q_out must not overlap q_in.
 *
 * A token whose page slot lies past its request's pages goes to
 * scratch_page when scratch_page >= 0 (CUDA-graph padding lanes,
 * scheduler.py:366-369), else it is skipped and flagged.
 * ------------------------------------------------------------------------- */
int mi_append_paged_kv_cache(
    const void *append_key, int64_t k_stride_n, int64_t k_stride_h,
    const void *append_value, int64_t v_stride_n, int64_t v_stride_h,
    const int32_t *batch_indices, const int32_t *positions, int32_t nnz,
    void *kv_data, int64_t num_pages, int32_t page_size, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype,
    const int32_t *kv_indices, const int32_t *kv_indptr, int32_t batch_size,
    const void *rope_cos, const void *rope_sin, int32_t rope_max_pos,
    const int32_t *rope_positions,
    const void *q_in, int64_t q_in_stride_n, int64_t q_in_stride_h,
    void *q_out, int64_t q_out_stride_n, int64_t q_out_stride_h, int32_t num_qo_heads,
    int32_t scratch_page, int32_t *status, mi_stream_t stream);

/* ---------------------------------------------------------------------------
 * (2) Paged decode attention
 *
 * Replaces BatchDecodeWithPagedKVCacheWrapper.plan()/.run() as
 * scheduler.py:535-539, :905-916 and model.py:224-235 use it:
 *   out[b][h] = softmax(q[b][h] . K_b^T * sm_scale) . V_b
 * over the kv_len tokens of request b, query head h reading KV head
 * h / (num_qo_heads/num_kv_heads): native GQA for any group size, no head
 * padding (model.py:227-243 pads to a power of two; not needed here).
 * q: [batch][num_qo_heads][head_dim] with the given strides (elements);
 * out: contiguous [batch][num_qo_heads][head_dim] in `dtype`;
 * lse (optional): [batch][num_qo_heads] fp32, natural log. A request with
 * no tokens gets zeros and lse = -inf.
 *
 * The workspace holds split-K partial results and counters. It must be
 * zero-filled once before its first use; every call leaves its counters at
 * zero again (after an MI_STATUS_TIMEOUT, zero-fill it again). Calls sharing
 * a workspace must not overlap on the GPU. A page id outside the pool is
 * flagged (MI_STATUS_BAD_PAGE) and its tokens are left out.
 * ------------------------------------------------------------------------- */
size_t mi_paged_decode_workspace_size(int32_t batch_size, int32_t num_qo_heads,
                                      int32_t num_kv_heads, int32_t head_dim);
int mi_paged_decode(
    const void *q, int64_t q_stride_b, int64_t q_stride_h,
    const void *kv_data, int64_t num_pages, int32_t page_size, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype,
    const int32_t *kv_indptr, const int32_t *kv_indices, const int32_t *kv_last_page_len,
    int32_t batch_size, int32_t num_qo_heads, float sm_scale,
    void *out, float *lse, void *workspace, size_t workspace_bytes, int32_t *status,
    mi_stream_t stream);

/* ---------------------------------------------------------------------------
 * Decode step with the append fused in (no single FlashInfer counterpart:
 * it replaces the pair model.py:207-216 append_paged_kv_cache +
 * model.py:235 run of a decode step).
 *
 * Each request b has one new token at position kv_len_b - 1 (kv_len from
 * kv_indptr / kv_last_page_len, which already count it, as the reference's
 * decode-step page table does, scheduler.py:862). k_new / v_new:
 * [batch][num_kv_heads][head_dim], raw K (before RoPE) and V; q: raw
 * queries. The call writes K rotated by RoPE at that position (the append's
 * three roundings, model.py:92-107) and V into the token's page slot, and
 * computes mi_paged_decode over the rotated q. Result and pages are bit for
 * bit those of mi_append_paged_kv_cache(k_new, v_new, batch_indices =
 * 0..batch-1, positions = kv_len - 1, rope tables, q_in = q, q_out)
 * followed by mi_paged_decode(q_out), in one launch pair. rope_cos /
 * rope_sin: [rope_max_pos][head_dim] in `dtype`; a position outside the
 * table is flagged MI_STATUS_BAD_POSITION and left out. Rows and tables
 * 16-byte aligned, strides multiples of 8 elements. Shapes outside the
 * stream-K decode kernel (fp32, head_dim other than 64/128, group > 16,
 * 1/2/4/8 KV heads only) return MI_ERR_UNSUPPORTED and launch nothing; the
 * caller then makes the two calls. The launch may start before the kernel
 * issued just before it on `stream` has finished (programmatic dependent
 * launch) and reads kv_data from the start: that kernel must not write
 * kv_data (a GEMM producing q / k_new / v_new is fine; an append into the
 * same pool is not).
 * ------------------------------------------------------------------------- */
int mi_paged_decode_append(
    const void *q, int64_t q_stride_b, int64_t q_stride_h,
    const void *k_new, int64_t k_stride_b, int64_t k_stride_h,
    const void *v_new, int64_t v_stride_b, int64_t v_stride_h,
    const void *rope_cos, const void *rope_sin, int32_t rope_max_pos,
    void *kv_data, int64_t num_pages, int32_t page_size, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype,
    const int32_t *kv_indptr, const int32_t *kv_indices, const int32_t *kv_last_page_len,
    int32_t batch_size, int32_t num_qo_heads, float sm_scale,
    void *out, float *lse, void *workspace, size_t workspace_bytes, int32_t *status,
    mi_stream_t stream);

/* ---------------------------------------------------------------------------
 * Paged decode for callers that cannot allocate device memory.
 *
 * No counterpart in the reference. Some hosts manage all GPU memory through
 * their own allocator (a serving runtime's caching pool, a fixed arena given
 * to plugins) and offer a kernel library no way to get a workspace; others
 * call from places where cudaMalloc is not allowed or would stall the
 * device. This variant of mi_paged_decode takes the same arguments minus the
 * workspace and allocates nothing: its split-K scratch is a fixed array of
 * MI_DECODE_STATIC_SCRATCH_BYTES inside the library, which every GPU that
 * loads the library holds until the process exits. The caller still passes
 * q, the pool, the page tables and out.
 *   - Limit: batch_size * num_kv_heads counters plus one partial slot per
 *     (request, KV head) of group*head_dim*4 bytes must fit in the array;
 *     larger calls return MI_ERR_WORKSPACE and launch nothing. The limit
 *     applies only to calls that the split-K kernels serve (16-bit dtypes,
 *     head_dim 64/128, group <= 16, batch <= 2048, 16-byte aligned rows);
 *     other calls run the generic kernel, which uses no scratch.
 *   - All calls share the array. Each call first clears its counters on
 *     `stream`; calls that overlap on the GPU (other streams, unordered
 *     threads) race on the array and must be serialised by the caller.
 *   - The first call on each device looks up the array's device address
 *     (with that device current) and caches it with the device's context;
 *     after a device reset the next call looks it up again. Make the first
 *     call on a device before any stream capture.
 * ------------------------------------------------------------------------- */
#define MI_DECODE_STATIC_SCRATCH_BYTES (8u << 20)
int mi_paged_decode_noalloc(
    const void *q, int64_t q_stride_b, int64_t q_stride_h,
    const void *kv_data, int64_t num_pages, int32_t page_size, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype,
    const int32_t *kv_indptr, const int32_t *kv_indices, const int32_t *kv_last_page_len,
    int32_t batch_size, int32_t num_qo_heads, float sm_scale,
    void *out, float *lse, int32_t *status, mi_stream_t stream);

/* ---------------------------------------------------------------------------
 * (3) Paged prefill attention
 *
 * Replaces BatchPrefillWithPagedKVCacheWrapper.plan()/.run() as
 * scheduler.py:530-534, :704-716 and model.py:219-235 use it: ragged
 * queries q[total_q][num_qo_heads][head_dim] split by qo_indptr[batch+1],
 * attending to each request's pages (appended first). With causal != 0,
 * query i of a request with qo_len queries and kv_len keys sees keys
 * j <= kv_len - qo_len + i. out: contiguous [total_q][num_qo_heads][head_dim];
 * lse optional as for decode. The workspace (mi_paged_prefill_workspace_size()
 * bytes, 16-byte aligned) holds the work-item counters the persistent
 * tensor-core kernel shares between its CTAs: zero-fill it once before its
 * first use; every call leaves it at zero again (after MI_STATUS_TIMEOUT,
 * zero-fill it again), and calls sharing a workspace must not overlap on the
 * GPU. Without a workspace (NULL or smaller) the kernel assigns work items
 * round robin instead.
 * ------------------------------------------------------------------------- */
size_t mi_paged_prefill_workspace_size(int32_t total_q, int32_t batch_size,
                                       int32_t num_qo_heads, int32_t head_dim);
int mi_paged_prefill(
    const void *q, int64_t q_stride_n, int64_t q_stride_h,
    const int32_t *qo_indptr, int32_t total_q,
    const void *kv_data, int64_t num_pages, int32_t page_size, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype,
    const int32_t *kv_indptr, const int32_t *kv_indices, const int32_t *kv_last_page_len,
    int32_t batch_size, int32_t num_qo_heads, int32_t causal, float sm_scale,
    void *out, float *lse, void *workspace, size_t workspace_bytes, int32_t *status,
    mi_stream_t stream);

/* ---------------------------------------------------------------------------
 * (4) Device page pool (replaces PagedKVCache's free list, scheduler.py:168-221)
 *
 * free_ring[num_pages] and pool_ctrl[4] are caller-owned device int32
 * buffers. The pool hands out pages 0..num_pages-2 in FIFO order; page
 * num_pages-1 is the scratch page and is never handed out (:204-206).
 * Allocation pops from the head, release appends to the tail (:208-221), so
 * page tables come out exactly as the reference's.
 * ------------------------------------------------------------------------- */
int mi_page_pool_init(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                      mi_stream_t stream);
/* Pop counts[0] + ... + counts[n-1] pages (all or nothing) into out_pages, in
 * request order (PagedKVCache.allocate_pages, scheduler.py:208-214). */
int mi_page_alloc(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                  const int32_t *counts, int32_t n, int32_t *out_pages,
                  int32_t *status, mi_stream_t stream);
/* Zero pages[0..n) in every layer, then append them to the free list in order
 * (PagedKVCache.release_pages, scheduler.py:216-221) -- one launch for all
 * pages and layers. layer_pools: device array of num_layers pool pointers;
 * page_bytes = 2*page_size*num_kv_heads*head_dim*elem_size. */
int mi_page_release(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                    const int32_t *pages, int32_t n, void *const *layer_pools,
                    int32_t num_layers, int64_t page_bytes, int32_t *status,
                    mi_stream_t stream);

/* Slot page tables: page_table[max_slots][max_pages_per_slot] and
 * slot_num_pages[max_slots] (device int32) hold the pages of each request
 * slot, so a CUDA graph can grow, read and release them without the host.
 * Slot ids outside [0, max_slots) are flagged (MI_STATUS_BAD_BATCH_INDEX) and
 * ignored; slots listed in one call must be distinct. */

/* Admission: pop counts[i] pages for slots[i], i = 0..n-1 in order
 * (scheduler.py:624-637). All or nothing. */
int mi_slot_alloc(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                  int32_t *page_table, int32_t *slot_num_pages, int32_t max_slots,
                  int32_t max_pages_per_slot,
                  const int32_t *slots, const int32_t *counts, int32_t n,
                  int32_t *status, mi_stream_t stream);
/* Retire: zero and free every page of slots[0..n) in order (pages of a slot in
 * allocation order), set their page counts to 0 (scheduler.py:984-1003). */
int mi_slot_release(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                    int32_t *page_table, int32_t *slot_num_pages, int32_t max_slots,
                    int32_t max_pages_per_slot,
                    const int32_t *slots, int32_t n, void *const *layer_pools,
                    int32_t num_layers, int64_t page_bytes, int32_t *status,
                    mi_stream_t stream);
/* One decode (or prefill) step's page metadata, on the device.
 * Lane i is request slot lane_slots[i] (-1: padding lane) whose newest token
 * sits at lane_positions[i]. With grow != 0, a lane whose slot holds fewer
 * than ceil((pos+1)/page_size) pages first pops the missing pages, lanes in
 * order (scheduler.py:842-847). Then writes the CSR page table of all
 * num_lanes lanes (scheduler.py:861-868): kv_indptr[num_lanes+1],
 * kv_indices (capacity indices_capacity), kv_last_page_len[num_lanes], and
 * append_positions[num_lanes] (pos, 0 for padding). Padding lanes get 0 pages
 * and last_page_len 1 (scheduler.py:887-896); their append goes to the
 * scratch page. */
int mi_step_prepare(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                    int32_t *page_table, int32_t *slot_num_pages, int32_t max_slots,
                    int32_t max_pages_per_slot,
                    const int32_t *lane_slots, const int32_t *lane_positions, int32_t num_lanes,
                    int32_t page_size, int32_t grow,
                    int32_t *kv_indptr, int32_t *kv_indices, int32_t indices_capacity,
                    int32_t *kv_last_page_len, int32_t *append_positions,
                    int32_t *status, mi_stream_t stream);

/* ---- decode-step glue (model.py:115-122, :301-311, :333-343) ---------- */

/* residual[r] = residual[r] + x[r] (rounded to dtype; skipped when x is
 * NULL), then out[r] = rms_norm(residual[r]) * weight with fp32 statistics:
 * the reference's `h = h + sublayer(...)` followed by F.rms_norm
 * (model.py:115-122, :333-343) in one launch. Rows are contiguous
 * [rows, hidden]; residual is updated in place; out must not alias it. */
int mi_add_rmsnorm(const void *x, void *residual, const void *weight, void *out,
                   int32_t rows, int32_t hidden, float eps, int32_t dtype,
                   mi_stream_t stream);

/* out[r, :] = silu(gate_up[r, :inter]) * gate_up[r, inter:] for contiguous
 * [rows, 2*inter] input (the fused gate/up GEMM output): the reference's
 * `F.silu(gate_proj(x)) * up_proj(x)` (model.py:311). */
int mi_silu_mul(const void *gate_up, void *out, int32_t rows, int32_t inter, int32_t dtype,
                mi_stream_t stream);

/* y[r, :] = x[r, :] w^T (+ bias) for m <= 32 rows: the reference's
 * nn.Linear projections (model.py:127-131, :306-308) at decode batch sizes,
 * where the weight is streamed once from HBM. x [m, k] (row stride ldx),
 * w [n, k] (row stride ldw; the nn.Linear layout), y [m, n] (row stride
 * ldy), bias [n] or NULL; bf16 / fp16 with fp32 accumulation, one rounding
 * at the end; k a multiple of 64; pointers 16-byte aligned, ldx / ldw
 * multiples of 8. Deterministic: K-split partial sums are added in a fixed
 * order. No workspace; m = 0 launches nothing. */
int mi_proj_small_m(const void *x, int64_t ldx, const void *w, int64_t ldw, const void *bias,
                    void *y, int64_t ldy, int32_t m, int32_t n, int32_t k, int32_t dtype,
                    int32_t *status, mi_stream_t stream);

/* ---- tensor parallelism: fused all-reduce for decode steps --------------- */

/* No FlashInfer counterpart: replaces, for decode-sized row counts, the
 * torch.distributed all_reduce after a row-parallel o_proj / down_proj plus
 * the residual add and RMSNorm that follow it (model.py:115-122, :333-343).
 *
 * Every rank owns a symmetric buffer (same size; each rank's buffer mapped
 * into every rank's address space); peer_bases[q] (a device array of
 * `world` 64-bit addresses) is rank q's buffer as this process sees it. At
 * byte offset data_off every rank's GEMM has written its partial
 * [rows][hidden] sum before this call; at flag_off lies a uint32 array
 * [world][256], zero-filled on every rank (and all ranks past a barrier)
 * before the first call. block_counters: this rank's uint32 [256], zeroed
 * once. Then: residual[r] += sum over ranks of partial[r] (rounded to dtype
 * as the all-reduce result, then as the add), out[r] = rms_norm(residual[r])
 * * weight. rows <= 256. Every rank must make the same sequence of calls
 * (same rows); a call site's partial must not be rewritten before this
 * rank's next call has returned. Waits for peers are bounded (10 s by
 * default, see mi_set_peer_wait_limit_ns): on give-up MI_STATUS_TIMEOUT is
 * set and the outputs are not written. */
int mi_allreduce_add_rmsnorm(const unsigned long long *peer_bases, int64_t data_off,
                             int64_t flag_off, uint32_t *block_counters, int32_t rank,
                             int32_t world, void *residual, const void *weight, void *out,
                             int32_t rows, int32_t hidden, float eps, int32_t dtype,
                             int32_t *status, mi_stream_t stream);

/* Give-up limit (nanoseconds of GPU wall time) of the peer barrier in
 * mi_allreduce_add_rmsnorm launches made after this call, process-wide;
 * ns <= 0 restores the default of 10 s. No reference counterpart: a
 * serving process lowers it to learn of a dead peer sooner. */
int mi_set_peer_wait_limit_ns(int64_t ns);

/* Peer mappings of the symmetric buffer (set-up calls, not for the hot
 * path; no reference counterpart). Plain CUDA IPC: the peer's allocation is
 * mapped over NVLink P2P and nothing is bound to an NVLink multicast object.
 * mi_ipc_export: handle (MI_IPC_HANDLE_BYTES bytes) of the cudaMalloc
 * allocation holding `ptr`, and ptr's byte offset in it. mi_ipc_open (in
 * another process): map that allocation, *base_out = its base address here
 * (add the offset). mi_ipc_close: unmap a base returned by mi_ipc_open. */
#define MI_IPC_HANDLE_BYTES 64
int mi_ipc_export(const void *ptr, void *handle_out, int64_t *offset_out);
int mi_ipc_open(const void *handle, void **base_out);
int mi_ipc_close(void *base);

#ifdef __cplusplus
}
#endif

#endif /* MI_PAGED_H */
