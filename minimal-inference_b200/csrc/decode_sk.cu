// Kernel (2), stream-K version: paged decode attention fed by TMA tensor loads.
//
// Same contract as decode.cu (FlashInfer BatchDecodeWithPagedKVCacheWrapper
// as scheduler.py:535-539, :905-916 and model.py:235 use it), for the shapes
// the reference serves: bf16/fp16, head_dim 64/128, page_size a multiple of
// 16, 1/2/4/8 KV heads, GQA group <= 16.
//
// Work split ("stream-K"): the requests' pages, concatenated in kv_indices
// order, are cut into gridDim.x equal runs of T = ceil(total/grid) pages;
// CTA i streams run i. A request wholly inside one run is finished there;
// one cut by run boundaries gets a normalised partial per run (slot
// blockIdx.x + b), which a second, fully parallel kernel merges (one warp
// per request and query head). Merging in the decode kernel itself put every
// merge at the very end of the runs, serialised behind the last arrivals.
// Both kernels derive T from kv_indptr on the device, so the launches need
// no host plan() and can be graph-captured.
//
// CTA = 1 producer warp + 8 consumer warps.
//   * Producer: walks its run in stages of up to tps = 8/Hkv consecutive
//     16-token tiles (so a stage is 64 KB at head_dim 128 whatever the KV
//     head count; fewer tiles only where shared memory is short). Page ids
//     come from coalesced 32-wide windows of kv_indices held in registers
//     (the next window is prefetched). For each stage it waits for a free
//     slot, writes the stage record, and its lanes issue one 4-D TMA tensor
//     load (cp.async.bulk.tensor, SWIZZLE_128B) per (tile, K/V, 64-wide half
//     of head_dim): a 16-token x Hkv-head x 128-byte box, laid out in shared
//     memory as [head][token][128 bytes] (with one KV head, one 5-D box per
//     tile). The stage's mbarrier counts the bytes. Whole-head boxes matter:
//     with one box per head the TMA issue rate, not HBM, bounded the kernel
//     (config 2: 60.7 us per launch with 32 boxes per tile, 52.9 with 4).
//   * Consumers: warp w serves KV head w / (8/Hkv); the 8/Hkv warps of a
//     head take turns over the tiles of a segment, one tile per stage at
//     most. The group's query heads are the M
//     rows of mma.sync m16n8k16 (S = Q K^T, O += P V, P in registers), online
//     softmax in the exp2 domain. The 128-byte swizzle puts the 8 rows of
//     every ldmatrix in different banks.
//   * Warps sharing a KV head combine through one shared-memory buffer: all
//     write (hsync), then each combines its share of the query rows and
//     releases the buffer (hdone) before any may write the next segment's
//     partials. All cross-warp waits are bounded, so nothing can hang.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "mi_common.cuh"

#include "decode_sk.cuh"
#include "tma.cuh"

namespace mi {
namespace {

constexpr int kNC = 8;                    // consumer warps
constexpr int kThreads = (kNC + 1) * 32;  // + one producer warp
constexpr int kTile = 16;
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 232448;        // 227 KB opt-in per CTA
constexpr size_t kCtrl = 256;
// Stream-K split: what a request start inside a run costs its CTA, in bytes
// of page stream. A segment boundary stalls the CTA's consumers for ~3.5 us
// (the previous segment's combine, the next one's query loads), about 154 KB
// of one SM's share of HBM bandwidth. Measured on a B200: with 8 KV heads a
// run shortened by k pages does not finish k pages' time sooner, and config
// 2's fused step (B=32) took 52.6 / 51.3 / 51.3 / 51.7 us per launch pair at
// 154 / 300 / 450 / 650 KB; with 1-4 KV heads (tensor-parallel and
// head-sharded shapes, B=32 and 64) 154 KB stayed within 3.3 % of the best
// of 0 / 60 / 154 / 380 KB on every shape, and 380 KB lost up to 13 %.
constexpr double kSegCostBytesWide = 380e3;  // 8 or more KV heads
constexpr double kSegCostBytes = 154e3;      // fewer

inline size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

struct SkParams {
  const void *q;
  int64_t qsb, qsh;
  int64_t num_pages;
  int ps, group, hq, batch, stages, stage_bytes, tps;  // KV heads: the kernel's HKV
  const int32_t *indptr, *indices, *last;
  float scale_log2;
  void *out;
  float *lse;
  int32_t *status;
  float *part_o;     // [(grid + batch)][hq][D]
  float *part_lse;   // [(grid + batch)][hq]
  int bar_off, rec_off, scr_off;
  int meta_off;  // >= 0: kv_indptr / kv_last_page_len staged in shared memory here
  int rope_off;  // per consumer warp: the RoPE cos and sin rows of its segment's position
  int seg_cost4;  // stream-K split: cost of a request start, in quarter pages (vsplit_run)
  // Fused append (mi_paged_decode_append; k_new == nullptr: plain decode):
  // request b's new token sits at position kv_len_b - 1. Its raw K is
  // rotated like the append kernel's, K and V are written into their page
  // slot and patched into the stage that holds that slot; q is raw and is
  // rotated at the same position as it is loaded.
  const void *k_new, *v_new;
  int64_t ksb, ksh, vsb, vsh;
  const void *rope_cos, *rope_sin;
  int rope_max;
  void *kv;  // the pool, for the new tokens' page writes
};

constexpr int kSmemBatch = 1024;  // requests whose metadata fits the shared-memory copy

// A stage holds nt <= tps consecutive 16-token tiles of one run segment.
// flags: 1 first stage of the segment, 2 last, 4 direct (request wholly in
// this run), 8 the segment reaches the request's last token; bits 8-15
// per-tile bad-page mask; bits 16-19 nt; bits 20+ the
// stage's ordinal within the segment.
struct __align__(16) StageRec {
  int b, tok0, kvlen, flags;
};

// Cost-balanced stream-K split, in virtual units of a quarter page. Page j
// of a request b with n_b > 0 pages starts at virtual position
//     vs_b + c4 + 4 j,   vs_b = 4 (indptr[b] - indptr[0]) + c4 * (non-empty
//                                requests before b),
// so every request's start is charged c4 quarter pages: the time a CTA's
// consumers spend at a segment boundary (the previous segment's combine and
// the next one's query loads), during which that CTA streams nothing. CTA i
// owns the pages whose virtual start lies in [i R, (i+1) R), R =
// max(4, ceil(VT / G)), VT = 4 * total + c4 * (non-empty requests): with c4 = 0 the
// runs hold equal page counts, with c4 > 0 a CTA whose run holds more
// request starts gets fewer pages. Warp-cooperative (all 32 lanes); `ip`
// may be global or shared memory.
__device__ __forceinline__ int vsplit_total(const int32_t *ip, int B, int c4, int lane) {
  int nz = 0;
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    nz += __popc(__ballot_sync(0xffffffffu, b < B && ip[b + 1] > ip[b]));
  }
  return 4 * (ip[B] - ip[0]) + c4 * nz;
}

// Page position (counted from indptr[0]) of the first page whose virtual
// start is >= x.
__device__ __forceinline__ int vsplit_page(const int32_t *ip, int B, int c4, int x, int lane) {
  const int base0 = ip[0];
  int nzpre = 0, best_b = -1, best_s = 0;
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + lane;
    const int np = b < B ? ip[b + 1] - ip[b] : 0;
    const unsigned nzm = __ballot_sync(0xffffffffu, np > 0);
    const int vs = 4 * ((b < B ? ip[b] : ip[B]) - base0) +
                   c4 * (nzpre + __popc(nzm & ((1u << lane) - 1u)));
    const unsigned cand = __ballot_sync(0xffffffffu, np > 0 && vs <= x);
    if (cand) {
      const int l = 31 - __clz(cand);
      best_b = b0 + l;
      best_s = __shfl_sync(0xffffffffu, vs, l);
    }
    nzpre += __popc(nzm);
    if (__ballot_sync(0xffffffffu, b < B && vs > x)) break;  // later requests start past x
  }
  if (best_b < 0) return 0;
  const int local = x - best_s - c4;
  const int j = local <= 0 ? 0 : min(ip[best_b + 1] - ip[best_b], (local + 3) >> 2);
  return ip[best_b] - base0 + j;
}

// Run length R. At least one page (4 units), so every run between the first
// and the last run of a request holds a page of it and writes its partial.
__device__ __forceinline__ int vsplit_len(int vt, int G) { return max(4, cdiv(vt, G)); }

// This CTA's page range [lo, hi) (page positions from indptr[0]).
__device__ __forceinline__ void vsplit_run(const int32_t *ip, int B, int c4, int G, int cta,
                                           int lane, int *lo, int *hi) {
  const int vt = vsplit_total(ip, B, c4, lane);
  const int rv = vsplit_len(vt, G);
  const int x0 = min(vt, cta * rv), x1 = min(vt, x0 + rv);
  *lo = vsplit_page(ip, B, c4, x0, lane);
  *hi = vsplit_page(ip, B, c4, x1, lane);
}

template <typename T, int D, bool G16, int HKV>
__global__ void __launch_bounds__(kThreads, 1)
    decode_sk_kernel(const __grid_constant__ CUtensorMap tmap, const SkParams p) {
  constexpr int KS = D / 16, NT = D / 8, DH = D / 64;
  constexpr int SUBS = kNC / HKV;                         // consumer warps per KV head
  constexpr int kBlockBytes = HKV * kTile * 128;          // one (K/V, d-half) block of a tile
  constexpr int kTileBytes = 2 * DH * kBlockBytes;        // one 16-token tile of all heads
  // TMA boxes per tile: one per (K/V, d-half) covering all heads, or with a
  // single KV head one box for the whole tile (measured faster there, and
  // slower at 2 and 4 heads)
  constexpr bool kWholeTile = HKV == 1;
  constexpr int kBoxes = kWholeTile ? 1 : 2 * DH;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = p.stages;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.bar_off);
  uint64_t *empty = full + kMaxStages;
  uint64_t *hsync = empty + kMaxStages;  // [hkv] all warps of a head wrote the scratch
  uint64_t *hdone = hsync + 8;           // [hkv] all warps of a head have read it
  StageRec *recs = reinterpret_cast<StageRec *>(smem + p.rec_off);
  float *scratch = reinterpret_cast<float *>(smem + p.scr_off);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x, cta = blockIdx.x;

  if (threadIdx.x < S) {
    mbar_init(&full[threadIdx.x], 1);
    mbar_init(&empty[threadIdx.x], kNC);
  }
  if (threadIdx.x >= 32 && threadIdx.x < 32 + HKV) {
    mbar_init(&hsync[threadIdx.x - 32], SUBS);
    mbar_init(&hdone[threadIdx.x - 32], SUBS);
  }
  pdl_trigger();  // the merge kernel may get scheduled next to this grid
  // Launched with PDL, this grid may start while the kernel before it (the
  // append that writes this step's K/V and q) still runs. Everything up to
  // the pdl_wait() calls below reads only the page-table metadata
  // (kv_indptr / kv_indices / kv_last_page_len), which no kernel of this
  // library that triggers its dependents early writes, and in the fused
  // form the pool's pages; q, the outputs and the workspace are touched only
  // after pdl_wait().
  // The producer's first page-id window only needs this CTA's run start, so
  // its loads go out together with the metadata staging below.
  int pre_pw = -1, pre_pwn = -1;
  if (warp == kNC) {
    if (lane == 0)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
    const int b0 = p.indptr[0], tot = p.indptr[p.batch] - b0;
    int lo0, hi0;
    vsplit_run(p.indptr, p.batch, p.seg_cost4, gridDim.x, blockIdx.x, lane, &lo0, &hi0);
    pre_pw = (lo0 + lane < tot) ? p.indices[b0 + lo0 + lane] : -1;
    pre_pwn = (lo0 + 32 + lane < tot) ? p.indices[b0 + lo0 + 32 + lane] : -1;
  }
  // per-request metadata, read many times below: one coalesced copy to smem
  const int32_t *ip = p.indptr, *lp = p.last;
  if (p.meta_off >= 0) {
    int32_t *s_ip = reinterpret_cast<int32_t *>(smem + p.meta_off);
    int32_t *s_lp = s_ip + p.batch + 1;
    for (int i = threadIdx.x; i <= p.batch; i += blockDim.x) {
      s_ip[i] = p.indptr[i];
      if (i < p.batch) s_lp[i] = p.last[i];
    }
    ip = s_ip;
    lp = s_lp;
  }
  fence_mbar_init();
  __syncthreads();
  const int base0 = ip[0];
  const int total = ip[p.batch] - base0;
  int lo = 0, hi = 0;  // this CTA's pages (warp-cooperative split, every warp)
  vsplit_run(ip, p.batch, p.seg_cost4, G, cta, lane, &lo, &hi);

  constexpr int block_bytes = kBlockBytes;

  // L1 prefetch of the global rows a segment start of request b reads (see
  // seg_begin below), spread over the producer's lanes: 128-byte lines.
  auto prefetch_segment = [&](int b, int kvlen) {
    constexpr int kLineRow = D * static_cast<int>(sizeof(T)) / 128;  // lines per head row
    const char *qb = static_cast<const char *>(p.q) + static_cast<int64_t>(b) * p.qsb * sizeof(T);
    for (int li = lane; li < p.hq * kLineRow; li += 32)
      prefetch_l1(qb + (static_cast<int64_t>(li / kLineRow) * p.qsh * sizeof(T)) +
                  (li % kLineRow) * 128);
    if (p.k_new == nullptr) return;
    const int pos = kvlen - 1;
    if (pos < 0 || pos >= p.rope_max) return;
    const char *kb = static_cast<const char *>(p.k_new) + static_cast<int64_t>(b) * p.ksb * sizeof(T);
    const char *vb = static_cast<const char *>(p.v_new) + static_cast<int64_t>(b) * p.vsb * sizeof(T);
    for (int li = lane; li < 2 * HKV * kLineRow; li += 32) {
      const int which = li / (HKV * kLineRow), r = li % (HKV * kLineRow);
      const char *base = which ? vb : kb;
      const int64_t hs = (which ? p.vsh : p.ksh) * sizeof(T);
      prefetch_l1(base + (r / kLineRow) * hs + (r % kLineRow) * 128);
    }
    if (lane < 2 * kLineRow) {
      const char *tab = static_cast<const char *>(lane < kLineRow ? p.rope_cos : p.rope_sin);
      prefetch_l1(tab + static_cast<int64_t>(pos) * D * sizeof(T) + (lane % kLineRow) * 128);
    } else if (lane == 2 * kLineRow) {
      prefetch_l1(p.indices + ip[b] + pos / p.ps);
    }
  };

  // =========================== producer warp ==============================
  if (warp == kNC) {
    int k = 0;
    bool ok_run = true;
    const uint64_t policy = evict_first_policy();
    if (lo < hi) {
      int b = 0;
      {  // request holding global page position lo: last b with indptr[b]-base0 <= lo
        int l = 0, h = p.batch - 1;
        while (l < h) {
          const int mid = (l + h + 1) >> 1;
          if (ip[mid] - base0 <= lo) l = mid; else h = mid - 1;
        }
        b = l;
      }
      int wbase = lo;
      int pw = pre_pw, pwn = pre_pwn;  // loaded during the prologue
      // Plain decode: the predecessor may be the append that writes this
      // step's K/V, so its writes must be visible to the TMA loads first. The
      // fused form writes the step's K/V itself, and its predecessor must not
      // write the pool (the entry point's contract): the pages stream while
      // the predecessor (the previous layer's merge, or a GEMM) still runs.
      if (p.k_new == nullptr) pdl_wait();
      for (int pos = lo; pos < hi && ok_run;) {
        while (ip[b + 1] - base0 <= pos) ++b;
        const int start_b = ip[b] - base0, end_b = ip[b + 1] - base0;
        const int kvlen = kv_len_of(ip, lp, b, p.ps);
        const int sub_hi = min(hi, end_b);
        const bool direct = start_b >= lo && end_b <= hi;
        const int tok_begin = (pos - start_b) * p.ps;
        const int tok_end = min(kvlen, (sub_hi - start_b) * p.ps);
        // A segment without tokens (last_page_len 0) still gets one fully
        // masked tile, so its partial and its merge arrival exist.
        const int ntiles = tok_end > tok_begin ? cdiv(tok_end - tok_begin, kTile) : 1;
        for (int j0 = 0, ord = 0; j0 < ntiles; j0 += p.tps, ++ord) {
          const int nt = min(p.tps, ntiles - j0);
          const int tok0 = tok_begin + j0 * kTile;
          const int gpos0 = start_b + tok0 / p.ps;  // page position of the stage's first tile
          while (gpos0 >= wbase + 32) {
            wbase += 32;
            pw = pwn;
            pwn = (wbase + 32 + lane < total) ? p.indices[base0 + wbase + 32 + lane] : -1;
          }
          // lane -> (tile t, K/V, d-half); a stage spans at most 9 pages,
          // so its page ids sit in the current or the next window
          const int t = lane / kBoxes, r = lane % kBoxes;
          const int ttok = tok0 + t * kTile;
          int page;
          bool mine, bad;
          int badmask = 0;
          if constexpr (SUBS == 1) {  // one tile per stage, one page id for all lanes
            page = __shfl_sync(0xffffffffu, pw, gpos0 - wbase);
            mine = t < nt;
            bad = page < 0 || page >= p.num_pages;
            badmask = bad ? 1 : 0;
          } else {
            const int off = start_b + ttok / p.ps - wbase;
            const int pa = __shfl_sync(0xffffffffu, pw, off & 31);
            const int pb = __shfl_sync(0xffffffffu, pwn, off & 31);
            page = off < 32 ? pa : pb;
            mine = t < nt;
            bad = mine && (page < 0 || page >= p.num_pages);
            const unsigned badl = __ballot_sync(0xffffffffu, bad);
            for (int tt = 0; tt < nt; ++tt) badmask |= ((badl >> (tt * kBoxes)) & 1u) << tt;
          }
          // A later segment's first stage: the consumers will need the
          // request's query rows (and, fused, its new K / V rows, the RoPE
          // rows of its position and the new token's page id) when this
          // stage comes up, about S stages from now. Pull them into this
          // SM's L1 now, so that segment start does not stall all consumer
          // warps on loads queued behind the page stream. (The run's first
          // segment is loaded by the consumers right away.)
          if (j0 == 0 && pos != lo) prefetch_segment(b, kvlen);
          // everything but the issue itself is ready before the wait for a free slot
          const int s = k % S;
          const int flags = (j0 == 0 ? 1 : 0) | (j0 + nt >= ntiles ? 2 : 0) | (direct ? 4 : 0) |
                            (end_b <= hi ? 8 : 0) | (badmask << 8) | (nt << 16) |
                            ((ord & 2047) << 20);
          const uint32_t tx = static_cast<uint32_t>(nt - __popc(badmask)) * kTileBytes;
          const int dh = r % DH, which = r / DH;
          unsigned char *dst =
              smem + s * p.stage_bytes + t * kTileBytes + (which * DH + dh) * block_bytes;
          const int row = ttok % p.ps, plane = page * 2 + which;
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(&empty[s], ((k / S) & 1) ^ 1))) {
            ok_run = false;
            break;
          }
          if (lane == 0) {
            recs[s] = StageRec{b, tok0, kvlen, flags};
            mbar_arrive_expect_tx(&full[s], tx);
            if (badmask) flag(p.status, MI_STATUS_BAD_PAGE);
          }
          __syncwarp();
          if (mine && !bad) {
            if constexpr (kWholeTile)
              tma_load_5d(dst, &tmap, 0, row, 0, 0, plane, &full[s], policy);
            else
              tma_load_4d(dst, &tmap, dh * 64, row, 0, plane, &full[s], policy);
          }
          ++k;
        }
        pos = sub_hi;
      }
    }
    // end-of-run sentinel
    bool sentinel = false;
    if (ok_run) {
      const int s = k % S;
      if (__all_sync(0xffffffffu, mbar_wait_bounded(&empty[s], ((k / S) & 1) ^ 1))) {
        if (lane == 0) {
          recs[s] = StageRec{-1, 0, 0, 0};
          mbar_arrive(&full[s]);
        }
        sentinel = true;
      } else {
        ok_run = false;
      }
    }
    // No copy may still be in flight when the CTA retires. The sentinel
    // reused stage k % S, whose copy (issue k - S) had landed before its
    // consumers released it, so only the later issues need a wait.
    for (int kk = max(0, sentinel ? k - S + 1 : k - S); kk < k; ++kk)
      if (!mbar_wait_bounded(&full[kk % S], (kk / S) & 1)) ok_run = false;
    if (!ok_run && lane == 0) flag(p.status, MI_STATUS_TIMEOUT);
    return;
  }

  // =========================== consumer warps =============================
  pdl_wait();  // q, out, lse and the workspace are the predecessor's to finish with
  constexpr int subs = SUBS;
  const int h = warp / subs, sw = warp % subs;
  const int gid = lane >> 2, tq = lane & 3;

  // requests with no tokens: zeros, lse = -inf
  for (int b = cta * kNC + warp; b < p.batch; b += G * kNC) {
    if (kv_len_of(ip, lp, b, p.ps) != 0) continue;
    T *o = static_cast<T *>(p.out) + static_cast<int64_t>(b) * p.hq * D;
    for (int i = lane; i < p.hq * D; i += 32) o[i] = Elt<T>::from(0.f);
    if (p.lse)
      for (int i = lane; i < p.hq; i += 32) p.lse[b * p.hq + i] = -INFINITY;
  }

  uint32_t qa[KS][4];
  float o[NT][4];
  float m0 = -INFINITY, l0 = 0.f, m1 = -INFINITY, l1 = 0.f;
  int segments = 0;
  bool timed_out = false;
  // fused append: this lane's 16-byte chunk of the new token's K (rotated)
  // or V row of head h, patched into the stage that holds the token
  uint4 patch = make_uint4(0, 0, 0, 0);
  bool have_patch = false;
  constexpr int kChunks = D / 8;           // 16-byte chunks of a K or V row
  const int pw_which = lane / kChunks;     // lane -> (K or V, chunk)
  const int pw_cc = lane % kChunks;
  // this warp's copy of the RoPE cos / sin rows of the segment's position
  unsigned char *rope_sm = smem + p.rope_off + warp * (2 * D * static_cast<int>(sizeof(T)));

  // Start of a run segment of request b (kv_len tokens; has_new: the
  // segment holds the request's last token): this warp's query rows into
  // qa, rotated in the fused form, and the fused append's K / V chunk into
  // `patch` with the token's page write. Every global load is issued before
  // any of them is used, so a segment start costs one round trip.
  auto seg_begin = [&](int b, int kvlen, bool has_new) {
    const T *qb = static_cast<const T *>(p.q) + static_cast<int64_t>(b) * p.qsb;
    const int r0 = h * p.group + gid;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      const int dc = kk * 16 + 2 * tq;
      uint32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
      if (gid < p.group) {
        const T *qr = qb + static_cast<int64_t>(r0) * p.qsh;
        a0 = *reinterpret_cast<const uint32_t *>(qr + dc);
        a2 = *reinterpret_cast<const uint32_t *>(qr + dc + 8);
      }
      if (G16 && gid + 8 < p.group) {
        const T *qr = qb + static_cast<int64_t>(r0 + 8) * p.qsh;
        a1 = *reinterpret_cast<const uint32_t *>(qr + dc);
        a3 = *reinterpret_cast<const uint32_t *>(qr + dc + 8);
      }
      qa[kk][0] = a0;
      qa[kk][1] = a1;
      qa[kk][2] = a2;
      qa[kk][3] = a3;
    }
    have_patch = false;
    if (p.k_new == nullptr) return;
    // fused append: the request's new token is its last, at kv_len - 1
    const int pos = kvlen - 1;
    const bool rope_ok = pos >= 0 && pos < p.rope_max;
    const T *cr = static_cast<const T *>(p.rope_cos) + static_cast<int64_t>(rope_ok ? pos : 0) * D;
    const T *sr = static_cast<const T *>(p.rope_sin) + static_cast<int64_t>(rope_ok ? pos : 0) * D;
    // the position's cos and sin rows (D/4 chunks of 16 bytes), staged in
    // this warp's shared-memory slot below
    uint4 csv = make_uint4(0, 0, 0, 0);
    if (rope_ok && lane < D / 4)
      csv = *reinterpret_cast<const uint4 *>(lane < D / 8 ? cr + lane * 8 : sr + (lane - D / 8) * 8);
    // the new token's K (rotated) or V chunk of head h: lane -> (K/V, chunk)
    const bool patch_lane = rope_ok && has_new && lane < 2 * kChunks;
    const int half = kChunks / 2, pc = pw_cc < half ? pw_cc + half : pw_cc - half;
    uint4 xv = make_uint4(0, 0, 0, 0), rv = xv;
    int page = -1;
    if (patch_lane) {
      if (pw_which == 0) {
        const T *kr = static_cast<const T *>(p.k_new) + static_cast<int64_t>(b) * p.ksb +
                      static_cast<int64_t>(h) * p.ksh;
        xv = *reinterpret_cast<const uint4 *>(kr + pw_cc * 8);
        rv = *reinterpret_cast<const uint4 *>(kr + pc * 8);
      } else {
        const T *vr = static_cast<const T *>(p.v_new) + static_cast<int64_t>(b) * p.vsb +
                      static_cast<int64_t>(h) * p.vsh;
        xv = *reinterpret_cast<const uint4 *>(vr + pw_cc * 8);
      }
      if (sw == 0) page = p.indices[ip[b] + pos / p.ps];
    }
    // ---- all loads issued; now the arithmetic ----
    if (!rope_ok) {
      if (lane == 0) flag(p.status, MI_STATUS_BAD_POSITION);  // left out, q unrotated
      return;
    }
    if (lane < D / 4) *reinterpret_cast<uint4 *>(rope_sm + lane * 16) = csv;
    __syncwarp();
    const T *cs_row = reinterpret_cast<const T *>(rope_sm);  // cos [0, D), sin [D, 2D)
    // all lanes keep the flag, so the stage patch runs warp-wide
    if (has_new) have_patch = true;
    if (patch_lane) {
      if (pw_which == 0) {
        const uint4 cv = *reinterpret_cast<const uint4 *>(cs_row + pw_cc * 8);
        const uint4 sv = *reinterpret_cast<const uint4 *>(cs_row + D + pw_cc * 8);
        const T *xe = reinterpret_cast<const T *>(&xv), *re = reinterpret_cast<const T *>(&rv);
        const T *ce = reinterpret_cast<const T *>(&cv), *se = reinterpret_cast<const T *>(&sv);
        T *pe = reinterpret_cast<T *>(&patch);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float r = Elt<T>::to(re[e]);
          pe[e] = Elt<T>::from(rope1<T>(Elt<T>::to(xe[e]), pw_cc < half ? -r : r,
                                        Elt<T>::to(ce[e]), Elt<T>::to(se[e])));
        }
      } else {
        patch = xv;
      }
      // one warp per head writes the token into its page slot
      if (sw == 0 && page >= 0 && page < p.num_pages) {
        T *dst = static_cast<T *>(p.kv) +
                 ((static_cast<int64_t>(page) * 2 + pw_which) * p.ps + pos % p.ps) * (HKV * D) +
                 h * D + pw_cc * 8;
        *reinterpret_cast<uint4 *>(dst) = patch;
      }
    }
    // q, after the patch (whose registers are free again): element d pairs
    // with d + D/2, held by this lane in k-step kk + KS/2; a lane's columns
    // in k-step kk are kk*16 + 2*tq + {0, 8} (+1)
#pragma unroll
    for (int kk = 0; kk < KS / 2; ++kk) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int d = kk * 16 + 2 * tq + ((i & 2) ? 8 : 0);
        const uint32_t cl = *reinterpret_cast<const uint32_t *>(cs_row + d);
        const uint32_t sl = *reinterpret_cast<const uint32_t *>(cs_row + D + d);
        const uint32_t ch = *reinterpret_cast<const uint32_t *>(cs_row + d + D / 2);
        const uint32_t sh = *reinterpret_cast<const uint32_t *>(cs_row + D + d + D / 2);
        const T *xl = reinterpret_cast<const T *>(&qa[kk][i]);
        const T *xh = reinterpret_cast<const T *>(&qa[kk + KS / 2][i]);
        const T *cle = reinterpret_cast<const T *>(&cl);
        const T *sle = reinterpret_cast<const T *>(&sl);
        const T *che = reinterpret_cast<const T *>(&ch);
        const T *she = reinterpret_cast<const T *>(&sh);
        uint32_t lo, hi;
        T *loe = reinterpret_cast<T *>(&lo), *hie = reinterpret_cast<T *>(&hi);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float x1 = Elt<T>::to(xl[e]), x2 = Elt<T>::to(xh[e]);
          loe[e] = Elt<T>::from(rope1<T>(x1, -x2, Elt<T>::to(cle[e]), Elt<T>::to(sle[e])));
          hie[e] = Elt<T>::from(rope1<T>(x2, x1, Elt<T>::to(che[e]), Elt<T>::to(she[e])));
        }
        qa[kk][i] = lo;
        qa[kk + KS / 2][i] = hi;
      }
    }
  };

  // The first segment of this CTA's run is known before its first stage
  // lands (the producer derives it the same way): its loads go out now,
  // under the latency of the first TMA loads.
  int pre_b = -1;
  {
    if (lo < hi) {
      int l = 0, hb = p.batch - 1;
      while (l < hb) {
        const int mid = (l + hb + 1) >> 1;
        if (ip[mid] - base0 <= lo) l = mid; else hb = mid - 1;
      }
      while (ip[l + 1] - base0 <= lo) ++l;
      seg_begin(l, kv_len_of(ip, lp, l, p.ps), ip[l + 1] - base0 <= hi);
      pre_b = l;
    }
  }

  for (int k = 0;; ++k) {
    const int s = k % S;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (k / S) & 1))) {
      timed_out = true;
      break;
    }
    const StageRec rec = recs[s];
    if (rec.b < 0) break;
    const int flags = rec.flags;
    if (flags & 1) {  // first tile of a run segment: this warp's query rows
      if (rec.b != pre_b) seg_begin(rec.b, rec.kvlen, (flags & 8) != 0);
      pre_b = -1;
#pragma unroll
      for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
    }
    // this warp's tile of the stage: the head's warps take the segment's
    // tiles in turn (tile index ord * tps + t goes to warp (ord * tps + t) % subs)
    const int nt = (flags >> 16) & 15, ord = flags >> 20;
    const int t = subs == 1 ? 0 : (sw - (ord * p.tps) % subs + subs) % subs;
    if (t < nt) {
      unsigned char *st = smem + s * p.stage_bytes + t * kTileBytes;
      const uint32_t kbase = smem_u32(st) + h * (kTile * 128);
      const uint32_t vbase = kbase + DH * block_bytes;
      const int nvalid = ((flags >> (8 + t)) & 1) ? 0 : rec.kvlen - (rec.tok0 + t * kTile);
      if (nvalid < kTile) {
        // rows past the request (or of a bad page) may hold anything: zero
        // this head's V rows there so P = 0 never meets a NaN
        const int rows = kTile - max(nvalid, 0);
        unsigned char *vrow = st + DH * block_bytes + h * (kTile * 128);
        for (int idx = lane; idx < rows * 8 * DH; idx += 32) {
          const int dh = idx / (rows * 8), rem = idx % (rows * 8);
          const int r = max(nvalid, 0) + rem / 8, c = rem % 8;
          *reinterpret_cast<uint4 *>(vrow + dh * block_bytes + r * 128 + c * 16) =
              make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
        fence_proxy_async_smem();
      }
      if (have_patch) {
        // fused append: the stage loaded the page before this step's token
        // was written; put the new K / V row of head h in place
        const int rn = rec.kvlen - 1 - (rec.tok0 + t * kTile);
        if (rn >= 0 && rn < kTile) {
          if (lane < 2 * kChunks && nvalid > rn) {
            const int dh = pw_cc >> 3, c = pw_cc & 7;
            *reinterpret_cast<uint4 *>(st + (pw_which * DH + dh) * block_bytes +
                                       h * (kTile * 128) + swz(rn, c)) = patch;
          }
          __syncwarp();
          // the stage is refilled by TMA (async proxy) once released
          fence_proxy_async_smem();
          have_patch = false;
        }
      }
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
      {
        // even / odd k-steps accumulate separately: two MMA chains per n-tile
        float e0[4] = {0.f, 0.f, 0.f, 0.f}, e1[4] = {0.f, 0.f, 0.f, 0.f};
        const int mi = lane >> 3;
        const int rk = ((mi >> 1) << 3) + (lane & 7);  // token row of this lane's address
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          const int c = ((kk & 3) << 1) + (mi & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(b0, b1, b2, b3, kbase + (kk >> 2) * block_bytes + swz(rk, c));
          if (kk & 1) {
            Mma<T>::run(e0, qa[kk], b0, b1);
            Mma<T>::run(e1, qa[kk], b2, b3);
          } else {
            Mma<T>::run(s0, qa[kk], b0, b1);
            Mma<T>::run(s1, qa[kk], b2, b3);
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          s0[i] += e0[i];
          s1[i] += e1[i];
        }
      }
      auto ok = [&](int tok) { return tok < nvalid; };
      const int ta = 2 * tq, tb = 2 * tq + 1, tc = 8 + 2 * tq, td = 9 + 2 * tq;
      const float x0 = ok(ta) ? s0[0] * p.scale_log2 : -INFINITY;
      const float x1 = ok(tb) ? s0[1] * p.scale_log2 : -INFINITY;
      const float x2 = ok(tc) ? s1[0] * p.scale_log2 : -INFINITY;
      const float x3 = ok(td) ? s1[1] * p.scale_log2 : -INFINITY;
      float mx = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn0 = fmaxf(m0, mx);
      const float ms0 = mn0 == -INFINITY ? 0.f : mn0;
      const float corr0 = exp2f(m0 - ms0);
      const float p0 = exp2f(x0 - ms0), p1 = exp2f(x1 - ms0);
      const float p2 = exp2f(x2 - ms0), p3 = exp2f(x3 - ms0);
      l0 = l0 * corr0 + (p0 + p1 + p2 + p3);
      m0 = mn0;
      uint32_t pa[4];
      pa[0] = Mma<T>::pack(p0, p1);
      pa[2] = Mma<T>::pack(p2, p3);
      pa[1] = pa[3] = 0u;
      float corr1 = 1.f;
      if constexpr (G16) {
        const float y0 = ok(ta) ? s0[2] * p.scale_log2 : -INFINITY;
        const float y1 = ok(tb) ? s0[3] * p.scale_log2 : -INFINITY;
        const float y2 = ok(tc) ? s1[2] * p.scale_log2 : -INFINITY;
        const float y3 = ok(td) ? s1[3] * p.scale_log2 : -INFINITY;
        float my = fmaxf(fmaxf(y0, y1), fmaxf(y2, y3));
        my = fmaxf(my, __shfl_xor_sync(0xffffffffu, my, 1));
        my = fmaxf(my, __shfl_xor_sync(0xffffffffu, my, 2));
        const float mn1 = fmaxf(m1, my);
        const float ms1 = mn1 == -INFINITY ? 0.f : mn1;
        corr1 = exp2f(m1 - ms1);
        const float q0 = exp2f(y0 - ms1), q1 = exp2f(y1 - ms1);
        const float q2 = exp2f(y2 - ms1), q3 = exp2f(y3 - ms1);
        l1 = l1 * corr1 + (q0 + q1 + q2 + q3);
        m1 = mn1;
        pa[1] = Mma<T>::pack(q0, q1);
        pa[3] = Mma<T>::pack(q2, q3);
      }
      if (__any_sync(0xffffffffu, corr0 != 1.f || corr1 != 1.f)) {  // a row max moved
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          o[n][0] *= corr0;
          o[n][1] *= corr0;
          if constexpr (G16) {
            o[n][2] *= corr1;
            o[n][3] *= corr1;
          }
        }
      }
      {
        const int mi = lane >> 3;
        const int rv = ((mi & 1) << 3) + (lane & 7);
#pragma unroll
        for (int np = 0; np < KS; ++np) {
          const int c = ((np & 3) << 1) + (mi >> 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(b0, b1, b2, b3, vbase + (np >> 2) * block_bytes + swz(rv, c));
          Mma<T>::run(o[2 * np], pa, b0, b1);
          Mma<T>::run(o[2 * np + 1], pa, b2, b3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    if (!(flags & 2)) continue;
    // ---- end of a run segment: combine the warps of this KV head ----------
    // Before overwriting its scratch row block, a warp waits until all of
    // the head's warps have read the previous segment's.
    if (subs > 1 && segments > 0 &&
        !__all_sync(0xffffffffu, mbar_wait_bounded(&hdone[h], (segments - 1) & 1))) {
      timed_out = true;
      break;
    }
    ++segments;
    const int RS = p.group * (D + 2);  // floats per warp in the scratch
    float *mine = scratch + static_cast<size_t>(warp) * RS;
    {
      float ls0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
      ls0 += __shfl_xor_sync(0xffffffffu, ls0, 2);
      float ls1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
      ls1 += __shfl_xor_sync(0xffffffffu, ls1, 2);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        if (gid < p.group)
          *reinterpret_cast<float2 *>(mine + gid * (D + 2) + n * 8 + 2 * tq) =
              make_float2(o[n][0], o[n][1]);
        if (G16 && gid + 8 < p.group)
          *reinterpret_cast<float2 *>(mine + (gid + 8) * (D + 2) + n * 8 + 2 * tq) =
              make_float2(o[n][2], o[n][3]);
      }
      if (tq == 0) {
        if (gid < p.group) {
          mine[gid * (D + 2) + D] = m0;
          mine[gid * (D + 2) + D + 1] = ls0;
        }
        if (G16 && gid + 8 < p.group) {
          mine[(gid + 8) * (D + 2) + D] = m1;
          mine[(gid + 8) * (D + 2) + D + 1] = ls1;
        }
      }
    }
    __syncwarp();
    if (subs > 1) {
      if (lane == 0) mbar_arrive(&hsync[h]);
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&hsync[h], (segments - 1) & 1))) {
        timed_out = true;
        break;
      }
    }
    // warp (h, sw): rows h*group + r, r = sw, sw + subs, ... of request rec.b
    const int b = rec.b;
    const bool direct = flags & 4;
    constexpr int DPL = D / 32;
    const float *first = scratch + static_cast<size_t>(h * subs) * RS;
    const int slot = cta + b;
    for (int r = sw; r < p.group; r += subs) {
      float M = -INFINITY;
      for (int j = 0; j < subs; ++j) M = fmaxf(M, first[j * RS + r * (D + 2) + D]);
      float acc[DPL], L = 0.f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
      if (M != -INFINITY) {
        for (int j = 0; j < subs; ++j) {
          const float *row = first + j * RS + r * (D + 2);
          const float w = exp2f(row[D] - M);
          L += w * row[D + 1];
#pragma unroll
          for (int i = 0; i < DPL; ++i) acc[i] += w * row[i * 32 + lane];
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      const int qrow = h * p.group + r;
      if (direct) {
        T *ob = static_cast<T *>(p.out) + (static_cast<int64_t>(b) * p.hq + qrow) * D;
#pragma unroll
        for (int i = 0; i < DPL; ++i) ob[i * 32 + lane] = Elt<T>::from(acc[i] * inv);
        if (p.lse && lane == 0)
          p.lse[b * p.hq + qrow] = L > 0.f ? (M + __log2f(L)) * kLn2 : -INFINITY;
      } else {
        float *po = p.part_o + (static_cast<int64_t>(slot) * p.hq + qrow) * D;
#pragma unroll
        for (int i = 0; i < DPL; ++i) po[i * 32 + lane] = acc[i] * inv;
        if (lane == 0) p.part_lse[slot * p.hq + qrow] = L > 0.f ? M + __log2f(L) : -INFINITY;
      }
    }
    if (subs > 1) {  // this warp's reads are done: the scratch may be reused once all are
      __syncwarp();
      if (lane == 0) mbar_arrive(&hdone[h]);
    }
  }
  if (timed_out && lane == 0) flag(p.status, MI_STATUS_TIMEOUT);
}

// Split-K merge: one warp per (request, query head), two per CTA (small
// CTAs find room next to the decode CTAs sooner). Requests whose pages
// all fall in one CTA's run were finished by the decode kernel; for the
// others, combine the normalised partials of the runs that cover them
// (slots first_run + b .. last_run + b), lanes over head_dim. The run range
// comes from kv_indptr before the wait (metadata only); after it, the lse
// and the partial rows of up to kBatch runs are loaded in one round.
template <typename T, int D>
__global__ void __launch_bounds__(64) decode_sk_merge_kernel(const SkParams p, int grid_runs) {
  constexpr int DPL = D / 32;
  constexpr int kBatch = 8;  // runs whose partial rows are in flight together
  const int lane = threadIdx.x & 31;
  const int wid = blockIdx.x * 2 + (threadIdx.x >> 5);
  int b = 0, qrow = 0, slot0 = 0, nch = 0;
  if (wid < p.batch * p.hq) {
    b = wid / p.hq;
    qrow = wid % p.hq;
  }
  // the runs that cover request b under the decode kernel's split
  // (vsplit_run): page j starts at vs_b + c4 + 4 j, run r covers [r R, (r+1) R)
  {
    const int bb = wid < p.batch * p.hq ? b : 0;
    const int base0 = p.indptr[0];
    const int np = p.indptr[bb + 1] - p.indptr[bb];
    int nz_total = 0, nz_before = 0;
    for (int c0 = 0; c0 < p.batch; c0 += 32) {
      const int r = c0 + lane;
      const bool ne = r < p.batch && p.indptr[r + 1] > p.indptr[r];
      const unsigned m = __ballot_sync(0xffffffffu, ne);
      nz_total += __popc(m);
      const int rel = bb - c0;  // requests c0 .. bb-1 of this chunk come before bb
      nz_before += rel >= 32 ? __popc(m) : (rel > 0 ? __popc(m & ((1u << rel) - 1u)) : 0);
    }
    const int vt = 4 * (p.indptr[p.batch] - base0) + p.seg_cost4 * nz_total;
    if (wid < p.batch * p.hq && vt > 0 && np > 0) {
      const int rv = vsplit_len(vt, grid_runs);
      const int v0 = 4 * (p.indptr[bb] - base0) + p.seg_cost4 * nz_before + p.seg_cost4;
      const int first = v0 / rv;
      nch = (v0 + 4 * (np - 1)) / rv - first + 1;
      slot0 = first + b;
    }
  }
  pdl_wait();     // every partial of the decode grid is written and visible
  pdl_trigger();  // the next kernel may get scheduled; it waits for this grid itself
  if (nch <= 1) return;
  const float *lse_col = p.part_lse + static_cast<int64_t>(slot0) * p.hq + qrow;
  const float *o_col = p.part_o + (static_cast<int64_t>(slot0) * p.hq + qrow) * D + lane;
  const int64_t o_step = static_cast<int64_t>(p.hq) * D;  // one slot
  float M = -INFINITY, wsum = 0.f, acc[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
  for (int c0 = 0; c0 < nch; c0 += kBatch) {
    // lse of runs c0 .. c0+kBatch-1 (one lane each) and their rows, all in flight
    const int cl = c0 + lane;
    const float lc = (lane < kBatch && cl < nch) ? __ldcg(lse_col + static_cast<int64_t>(cl) * p.hq)
                                                 : -INFINITY;
    float v[kBatch][DPL];
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
#pragma unroll
      for (int i = 0; i < DPL; ++i)
        v[j][i] = (c0 + j < nch) ? __ldcg(o_col + (c0 + j) * o_step + i * 32) : 0.f;
    // running rescale to the batch's max (online softmax over batches)
    const float mb = warp_max(lc);
    const float mn = fmaxf(M, mb);
    if (mn == -INFINITY) continue;
    const float corr = exp2f(M - mn);  // 0 when M = -inf
    wsum *= corr;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] *= corr;
    M = mn;
    const float w = exp2f(lc - M);  // 0 for lanes without a run
    wsum += warp_sum(w);
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const float wj = __shfl_sync(0xffffffffu, w, j);
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] += wj * v[j][i];
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  T *ob = static_cast<T *>(p.out) + (static_cast<int64_t>(b) * p.hq + qrow) * D;
#pragma unroll
  for (int i = 0; i < DPL; ++i) ob[i * 32 + lane] = Elt<T>::from(acc[i] * inv);
  if (p.lse && lane == 0)
    p.lse[b * p.hq + qrow] = wsum > 0.f ? (M + __log2f(wsum)) * kLn2 : -INFINITY;
}

// ---------------------------------------------------------------------------
// host side: tensor maps (cached per pool), launch
// ---------------------------------------------------------------------------
struct SkLayout {
  int stages, stage_bytes, tps, bar_off, rec_off, scr_off, meta_off, rope_off, smem;
};

// Shared memory: stages of tps tiles, barriers (full/empty per stage,
// hsync/hdone per KV head), stage records, the combine scratch (one
// group x (D+2) fp32 block per consumer warp) and, for batches up to
// kSmemBatch, a copy of kv_indptr / kv_last_page_len. tps is the largest
// power of two <= 8/Hkv that still leaves three stages (two at the least).
bool sk_layout(int hkv, int d, int group, int batch, SkLayout *L) {
  const int subs = kNC / hkv;
  const int tile_bytes = 2 * hkv * kTile * d * 2;
  const int scr = kNC * group * (d + 2) * 4;
  const int meta = batch <= kSmemBatch ? ((2 * batch + 4) * 4 + 15) / 16 * 16 : 0;
  const int rope = kNC * 2 * d * 2;  // cos + sin row per consumer warp (16-bit types)
  const int ctrl = (2 * kMaxStages + 16) * 8 + kMaxStages * 16;
  const int fixed = 1024 /*align slack*/ + ctrl + scr + meta + rope;
  for (int min_stages = 3; min_stages >= 2; --min_stages) {
    for (int tps = subs; tps >= 1; tps >>= 1) {
      const int stage_bytes = tps * tile_bytes;
      int st = (kSmemLimit - fixed) / stage_bytes;
      if (st > kMaxStages) st = kMaxStages;
      if (st < min_stages) continue;
      L->tps = tps;
      L->stages = st;
      L->stage_bytes = stage_bytes;
      L->bar_off = st * stage_bytes;
      L->rec_off = L->bar_off + (2 * kMaxStages + 16) * 8;
      L->scr_off = L->rec_off + kMaxStages * 16;
      L->rope_off = L->scr_off + scr;
      L->meta_off = meta ? L->rope_off + rope : -1;
      L->smem = L->rope_off + rope + meta + 1024;
      return L->smem <= kSmemLimit;
    }
  }
  return false;
}

template <typename T, int D, bool G16, int HKV>
int launch_sk_t(const SkArgs &a, const CUtensorMap &map, const SkParams &p, int grid,
                int smem) {
  static std::atomic<unsigned long long> attr_set{0};
  if (smem_limit_once(attr_set, decode_sk_kernel<T, D, G16, HKV>, kSmemLimit) != cudaSuccess)
    return check_launch("decode_sk_kernel smem attribute");
  cudaError_t e = launch_pdl(decode_sk_kernel<T, D, G16, HKV>, dim3(grid), dim3(kThreads), smem,
                             a.stream, map, p);
  if (e != cudaSuccess) return fail(MI_ERR_CUDA, "decode_sk_kernel launch: %s", cudaGetErrorString(e));
  const int warps = a.batch * a.hq;
  e = launch_pdl(decode_sk_merge_kernel<T, D>, dim3((warps + 1) / 2), dim3(64), 0, a.stream, p,
                 grid);
  if (e != cudaSuccess)
    return fail(MI_ERR_CUDA, "decode_sk_merge_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("decode_sk_merge_kernel");
}

template <typename T, int D, bool G16>
int launch_sk_h(const SkArgs &a, const CUtensorMap &map, const SkParams &p, int grid, int smem) {
  switch (a.hkv) {
    case 1: return launch_sk_t<T, D, G16, 1>(a, map, p, grid, smem);
    case 2: return launch_sk_t<T, D, G16, 2>(a, map, p, grid, smem);
    case 4: return launch_sk_t<T, D, G16, 4>(a, map, p, grid, smem);
    default: return launch_sk_t<T, D, G16, 8>(a, map, p, grid, smem);
  }
}

}  // namespace

size_t decode_sk_workspace_bytes(int batch, int hq, int hkv, int d) {
  const size_t slots = static_cast<size_t>(num_sms()) + batch;
  return kCtrl + al256(size_t(batch) * hkv * 4) + al256(slots * hq * d * 4) +
         al256(slots * hq * 4);
}

// Returns -1 when the shape/arguments are outside this kernel's coverage.
int launch_decode_sk(const SkArgs &a) {
  if (!(a.dtype == MI_DTYPE_BF16 || a.dtype == MI_DTYPE_F16)) return -1;
  if (!(a.d == 64 || a.d == 128)) return -1;
  if (!(a.hkv == 1 || a.hkv == 2 || a.hkv == 4 || a.hkv == 8)) return -1;
  if (a.ps % kTile != 0 || a.ps > 256) return -1;
  const int group = a.hq / a.hkv;
  if (group > 16 || a.qsb % 2 || a.qsh % 2) return -1;
  if ((reinterpret_cast<uintptr_t>(a.kv) & 15) || (reinterpret_cast<uintptr_t>(a.q) & 3) ||
      (reinterpret_cast<uintptr_t>(a.ws) & 255))
    return -1;
  if (a.num_pages * 2 > (1LL << 31)) return -1;
  if (a.ws == nullptr || a.ws_bytes < decode_sk_workspace_bytes(a.batch, a.hq, a.hkv, a.d))
    return -1;
  SkLayout L;
  if (!sk_layout(a.hkv, a.d, group, a.batch, &L)) return -1;
  CUtensorMap map;
  const bool mapped = a.hkv == 1
                          ? pool_tile_tensor_map(a.kv, a.num_pages, a.ps, a.hkv, a.d, a.dtype, &map)
                          : pool_tensor_map(a.kv, a.num_pages, a.ps, a.hkv, a.d, a.dtype, &map, true);
  if (!mapped) return -1;
  const int grid = num_sms();
  unsigned char *w = static_cast<unsigned char *>(a.ws);
  const size_t slots = static_cast<size_t>(grid) + a.batch;
  SkParams p{};
  p.q = a.q;
  p.qsb = a.qsb;
  p.qsh = a.qsh;
  p.num_pages = a.num_pages;
  p.ps = a.ps;
  p.group = group;
  p.hq = a.hq;
  p.batch = a.batch;
  p.stages = L.stages;
  p.stage_bytes = L.stage_bytes;
  p.tps = L.tps;
  p.indptr = a.indptr;
  p.indices = a.indices;
  p.last = a.last;
  p.scale_log2 = a.sm_scale * kLog2e;
  p.out = a.out;
  p.lse = a.lse;
  p.status = a.status;
  // the workspace keeps decode.cu's layout: control, B*Hkv counters (used by
  // the fallback kernel), then the partials
  p.part_o = reinterpret_cast<float *>(w + kCtrl + al256(size_t(a.batch) * a.hkv * 4));
  p.part_lse = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(p.part_o) +
                                         al256(slots * a.hq * a.d * 4));
  p.bar_off = L.bar_off;
  p.rec_off = L.rec_off;
  p.scr_off = L.scr_off;
  p.meta_off = L.meta_off;
  p.rope_off = L.rope_off;
  {
    const double page_bytes = double(a.ps) * a.hkv * a.d * 2 * 2;
    const double c = 4.0 * (a.hkv >= 8 ? kSegCostBytesWide : kSegCostBytes) / page_bytes;
    p.seg_cost4 = static_cast<int>(c > 4096.0 ? 4096.0 : c + 0.5);
  }
  if (a.k_new != nullptr) {
    // fused append: 16-byte rows of the new K / V and of the RoPE tables
    const bool rows_ok =
        a.v_new && a.rope_cos && a.rope_sin && a.rope_max > 0 &&
        (reinterpret_cast<uintptr_t>(a.k_new) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(a.v_new) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(a.rope_cos) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(a.rope_sin) & 15) == 0 && a.ksb % 8 == 0 &&
        a.ksh % 8 == 0 && a.vsb % 8 == 0 && a.vsh % 8 == 0 &&
        (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 && a.qsb % 8 == 0 && a.qsh % 8 == 0;
    if (!rows_ok) return -1;
    p.k_new = a.k_new;
    p.v_new = a.v_new;
    p.ksb = a.ksb;
    p.ksh = a.ksh;
    p.vsb = a.vsb;
    p.vsh = a.vsh;
    p.rope_cos = a.rope_cos;
    p.rope_sin = a.rope_sin;
    p.rope_max = a.rope_max;
    p.kv = const_cast<void *>(a.kv);
  }
  const bool g16 = group > 8;
  if (a.dtype == MI_DTYPE_BF16) {
    if (a.d == 128)
      return g16 ? launch_sk_h<__nv_bfloat16, 128, true>(a, map, p, grid, L.smem)
                 : launch_sk_h<__nv_bfloat16, 128, false>(a, map, p, grid, L.smem);
    return g16 ? launch_sk_h<__nv_bfloat16, 64, true>(a, map, p, grid, L.smem)
               : launch_sk_h<__nv_bfloat16, 64, false>(a, map, p, grid, L.smem);
  }
  if (a.d == 128)
    return g16 ? launch_sk_h<__half, 128, true>(a, map, p, grid, L.smem)
               : launch_sk_h<__half, 128, false>(a, map, p, grid, L.smem);
  return g16 ? launch_sk_h<__half, 64, true>(a, map, p, grid, L.smem)
             : launch_sk_h<__half, 64, false>(a, map, p, grid, L.smem);
}

}  // namespace mi
