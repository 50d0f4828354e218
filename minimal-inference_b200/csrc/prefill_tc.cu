// Kernel (3), tensor-core path: paged prefill attention on tcgen05 / TMEM.
//
// Replaces the FlashInfer fa2 prefill the reference runs (mma.sync,
// scheduler.py:530-534, :704-716, model.py:235) for bf16/fp16, head_dim
// 64/128, page_size a multiple of 16.
//
// Work item = (request, KV head, 128 "packed" query rows): a row is a (query
// token, query head of the GQA group) pair, row = token * group + head, so one
// K/V tile feeds the whole group (Tq = 128 / group tokens per item). The grid
// is persistent, one CTA per SM; CTAs take items from a counter shared
// through the workspace (each request's heaviest query tiles first), so set-up
// (barriers, TMEM, the query-tile prefix) is paid once per SM and the next
// item's metadata, Q and K/V loads run under the current item. 14 warps:
//   warp 0  producer: TMA loads of the Q tile (3-D map over q) and of 128-token
//           K/V tiles straight from the pages (4-D pool map, 16-token boxes),
//           two K/V stages, 128-byte swizzle;
//   warp 1  MMA issuer (one thread): S = Q K^T into TMEM (M=128, N=128,
//           K=head_dim, both operands K-major), then O += P V into TMEM
//           (P K-major from TMEM, V MN-major from shared memory), tcgen05.commit to
//           mbarriers. S of tile j+1 is issued as soon as the softmax warps
//           hold S of tile j in registers, so it runs under their softmax;
//           P V of tile j follows once P is written;
//   warps 2-9  softmax, two halves of four warps (S columns and O columns
//           split between them): thread = TMEM lane = query row. Each KV
//           tile: load the S row, causal/length mask, online softmax in the
//           exp2 domain, write the bf16 P row into TMEM, rescale the O row in
//           TMEM only when the row max grew by more than 2^8; at the item's
//           end hand the row sums to the epilogue warps and go on;
//   warps 10-13 epilogue: normalise the finished item's O and store it while
//           the softmax warps work on the next item.
// TMEM: S in columns [0,128), P, two O buffers (items alternate, so one
// item's first products go in while the epilogue reads the previous one's O). Every wait
// is bounded; TMEM is freed on every path.
#include <algorithm>
#include <type_traits>

#include "prefill.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace mi {
namespace {

constexpr int kM = 128;       // packed query rows per CTA
constexpr int kN = 128;       // KV tokens per tile
constexpr int kThreadsP = 448;  // producer, MMA issuer, 2 x 4 softmax warps, 4 epilogue warps
constexpr int kMaxBatchTc = 1024;

template <int D> struct PfLayout {
  static constexpr int DH = D / 64;                   // 64-wide blocks of head_dim
  static constexpr int Q_BYTES = DH * kM * 128;       // [dh][row][64]
  static constexpr int K_BYTES = DH * kN * 128;       // [dh][token][64]
  static constexpr int V_BYTES = K_BYTES;
  // ring depths: Q buffers (items), K stages, V stages (tiles)
  static constexpr int NQ = 2, NK = 2, NV = 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + NQ * Q_BYTES;
  static constexpr int V_OFF = K_OFF + NK * K_BYTES;
  static constexpr int BAR_OFF = V_OFF + NV * V_BYTES;  // 31 mbarriers + tmem base
  static constexpr int ITEM_OFF = BAR_OFF + 256;       // 2 work-item records
  // row max exchange [2 tiles][2 halves][128]; per O buffer: row sums
  // [2][2 halves][128], row max [2][128] and the item's output record
  static constexpr int XCH_OFF = ITEM_OFF + 64;
  static constexpr int LSUM_OFF = XCH_OFF + 2 * 2 * kM * 4;
  static constexpr int MFIN_OFF = LSUM_OFF + 2 * 2 * kM * 4;
  static constexpr int EREC_OFF = MFIN_OFF + 2 * kM * 4;
  static constexpr int META_OFF = EREC_OFF + 2 * 16;
  // tiles_pre, qo_indptr, kv_indptr [batch+1] and kv_len [batch], in shared memory
  static constexpr int META_INTS = 4 * (kMaxBatchTc + 1);
  static constexpr int SMEM = META_OFF + META_INTS * 4 + 1024;
  // TMEM columns: S [0, 128) fp32; P [128, 192) as bf16 pairs (the A operand
  // of P V); two O buffers of head_dim columns from 192
  static constexpr int P_COL = kN;
  static constexpr int O_COL = kN + kN / 2;
  static constexpr int OB_STRIDE = D;
  static constexpr int TMEM_COLS = 512;
};

// One work item = (request b, KV head h, query tile t0): the item record the
// producer hands to the MMA and softmax warps through a two-slot ring.
struct __align__(16) PfItem {
  int b, h, t0, n_tiles;  // b < 0: no more items
  int q_start, lq, lk, page_base;
};

template <typename T, int D>
// 14 warps: four of them share one SM sub-partition's 16 K registers, so at
// most 128 registers per thread
__global__ void __launch_bounds__(kThreadsP, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kvmap, const PrefillParams p) {
  using L = PfLayout<D>;
  constexpr int DH = L::DH;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  uint64_t *q_full = bars + 0, *q_empty = bars + 2;  // per Q buffer (NQ <= 2)
  // K and V tiles ride separate rings: a K stage frees as soon as its QK^T is
  // done, so K loads run ahead of V loads (NK <= 3, NV <= 2)
  uint64_t *k_full = bars + 4, *k_empty = bars + 7, *v_full = bars + 10, *v_empty = bars + 12;
  uint64_t *s_full = bars + 14, *s_free = bars + 15, *p_full = bars + 16, *o_done = bars + 17;
  uint64_t *o_full = bars + 18, *o_free = bars + 20, *it_full = bars + 22, *it_empty = bars + 24;
  uint64_t *xch = bars + 26;  // the two softmax halves' row maxima
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 28);
  uint64_t *l_ready = bars + 29;  // per O buffer: the item's row sums are in shared memory
  PfItem *items = reinterpret_cast<PfItem *>(smem + L::ITEM_OFF);
  int *tiles_pre = reinterpret_cast<int *>(smem + L::META_OFF);
  int *s_qo = tiles_pre + (kMaxBatchTc + 1);       // qo_indptr
  int *s_ip = s_qo + (kMaxBatchTc + 1);            // kv_indptr
  int *s_lk = s_ip + (kMaxBatchTc + 1);            // kv length per request

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = p.group;
  const int tq = kM / g;        // query tokens per item
  const int m_used = tq * g;    // packed rows in use

  // ---- once per CTA: query-tile prefix over requests, barriers, TMEM ------
  // qo_indptr entries are clamped to [0, total_q] and a request whose range
  // ends before it starts gets no rows, so no output row at or past total_q
  // is ever written; such an indptr is flagged (query rows left out)
  auto qo_at = [&](int i) { return min(max(p.qo_indptr[i], 0), p.total_q); };
  for (int i = threadIdx.x; i <= p.batch; i += blockDim.x) {
    const int v = qo_at(i);
    if (blockIdx.x == 0 && (v != p.qo_indptr[i] || (i < p.batch && qo_at(i + 1) < v)))
      flag(p.status, MI_STATUS_BAD_POSITION);
    s_qo[i] = v;
    s_ip[i] = p.indptr[i];
    if (i < p.batch) s_lk[i] = kv_len_of(p.indptr, p.last, i, p.ps);
  }
  if (warp == 0) {  // tiles_pre[i] = sum over b < i of ceil(qo_len_b / tq)
    int carry = 0;
    if (lane == 0) tiles_pre[0] = 0;
    for (int base = 0; base < p.batch; base += 32) {
      const int bb = base + lane;
      int x = bb < p.batch ? cdiv(max(0, qo_at(bb + 1) - qo_at(bb)), tq) : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (bb < p.batch) tiles_pre[bb + 1] = carry + x;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < L::NQ; ++i) {
        mbar_init(&q_full[i], 1);
        mbar_init(&q_empty[i], 1);
      }
      for (int i = 0; i < L::NK; ++i) {
        mbar_init(&k_full[i], 1);
        mbar_init(&k_empty[i], 1);
      }
      for (int i = 0; i < L::NV; ++i) {
        mbar_init(&v_full[i], 1);
        mbar_init(&v_empty[i], 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&o_full[i], 1);
        mbar_init(&o_free[i], 4);   // the 4 epilogue warps
        mbar_init(&l_ready[i], 8);  // the 8 softmax warps
        mbar_init(&it_full[i], 1);
        mbar_init(&it_empty[i], 9);  // the MMA thread and the 8 softmax warps
      }
      mbar_init(s_full, 1);
      mbar_init(s_free, 8);
      mbar_init(p_full, 8);
      mbar_init(o_done, 1);
      mbar_init(xch, 8);
    }
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(L::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_mbar_init();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem;  // S: columns [0, 128); O buffers at 128 and 128 + kObStride
  const int n_items = tiles_pre[p.batch] * p.hkv;
  bool ok = true;

  if (warp == 0) {
    // ============================ producer ==================================
    const uint64_t pol_q = evict_last_policy(), pol_kv = evict_first_policy();
    int gt = 0, qc = 0;
    int k_ahead = -1;  // lane 0: the next item's index, taken once this item's K tiles are out
    for (int it = 0; ok; ++it) {
      // next item: a counter shared by all CTAs (heaviest query tiles of each
      // request first), or round robin without a workspace
      // next item: a counter shared by all CTAs (heaviest query tiles of each
      // request first), or round robin without a workspace; the counter is
      // read while the previous item's last V tiles were being issued
      int k = 0;
      if (lane == 0) {
        k = k_ahead >= 0 ? k_ahead
                         : (p.ctr ? static_cast<int>(atomicAdd(p.ctr, 1u)) : blockIdx.x + it * gridDim.x);
        k_ahead = -1;
      }
      k = __shfl_sync(0xffffffffu, k, 0);
      PfItem rec{-1, 0, 0, 0, 0, 0, 0, 0};
      if (k < n_items) {
        int lo = 0, hi = p.batch - 1;  // last b with tiles_pre[b] * hkv <= k
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (tiles_pre[mid] * p.hkv <= k) lo = mid; else hi = mid - 1;
        }
        const int b = lo, ntq = tiles_pre[b + 1] - tiles_pre[b];
        const int rem = k - tiles_pre[b] * p.hkv;
        rec.b = b;
        rec.h = rem / ntq;
        rec.t0 = (ntq - 1 - rem % ntq) * tq;
        rec.q_start = s_qo[b];
        rec.lq = s_qo[b + 1] - rec.q_start;
        rec.lk = s_lk[b];
        rec.page_base = s_ip[b];
        const int rows_tok = min(tq, rec.lq - rec.t0);
        const int lim_tok =
            p.causal ? min(rec.lk, rec.lk - rec.lq + rec.t0 + rows_tok) : rec.lk;
        rec.n_tiles = lim_tok > 0 ? cdiv(lim_tok, kN) : 0;
      }
      const int slot = it & 1;
      if (it >= 2 && !__all_sync(0xffffffffu, mbar_wait_bounded(&it_empty[slot], ((it >> 1) - 1) & 1))) {
        ok = false;
        break;
      }
      if (lane == 0) {
        items[slot] = rec;
        mbar_arrive(&it_full[slot]);
      }
      if (rec.b < 0) break;
      if (rec.n_tiles == 0) continue;
      // page ids of 16-token chunks, 32 per window (four tiles), the current
      // and the next window in registers; loaded before the Q wait below
      const int nchunk = rec.n_tiles * 8;
      auto load_win = [&](int w) -> int {
        const int c = w * 32 + lane;
        return c < nchunk && c * 16 < rec.lk ? p.indices[rec.page_base + (c * 16) / p.ps] : -1;
      };
      int pw = load_win(0), pwn = load_win(1);
      // Q tile into the single Q buffer once the previous item's last QK^T is done
      const int qb = qc % L::NQ;  // Q buffer of this item
      if (qc >= L::NQ &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(&q_empty[qb], ((qc / L::NQ) - 1) & 1))) {
        ok = false;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&q_full[qb], DH * m_used * 128);
        for (int dh = 0; dh < DH; ++dh)
          tma_load_3d(smem + L::Q_OFF + qb * L::Q_BYTES + dh * kM * 128, &qmap, dh * 64,
                      rec.h * g, rec.q_start + rec.t0, &q_full[qb], pol_q);
      }
      ++qc;
      // K or V (which) of tile j of this item, global tile index gtile; page
      // is this lane's chunk's page id (chunk lane / DH of the tile)
      auto issue = [&](int j, int gtile, int which, int page) -> bool {
        const int nst = which ? L::NV : L::NK;
        const int st = gtile % nst;
        uint64_t *full = which ? &v_full[st] : &k_full[st];
        uint64_t *empty = which ? &v_empty[st] : &k_empty[st];
        if (gtile >= nst &&
            !__all_sync(0xffffffffu, mbar_wait_bounded(empty, ((gtile / nst) - 1) & 1)))
          return false;
        const int tok_tile = j * kN;
        const int nvc = min(8, cdiv(rec.lk - tok_tile, 16));
        unsigned char *base = smem + (which ? L::V_OFF + st * L::V_BYTES : L::K_OFF + st * L::K_BYTES);
        if (which == 1 && gtile < L::NV && nvc < 8) {
          // V chunks past the request's end are multiplied by P = 0; on a
          // stage's first use they hold whatever shared memory held, so zero
          // them (later uses keep an earlier tile's finite values there)
          for (int dh = 0; dh < DH; ++dh) {
            uint4 *v = reinterpret_cast<uint4 *>(base + dh * (kN * 128) + nvc * 16 * 128);
            for (int i = lane; i < (8 - nvc) * 16 * 128 / 16; i += 32) v[i] = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();  // the zeros are visible to the tensor core
          __syncwarp();
        }
        if (lane == 0) mbar_arrive_expect_tx(full, nvc * DH * 2048);
        __syncwarp();
        const int c = min(lane / DH, 7), dh = lane % DH;
        if (lane < 8 * DH && c < nvc) {
          const bool bad = page < 0 || page >= p.num_pages;
          // a bad page id loads from page 0 (in bounds) and is flagged; its
          // keys still count, so the result is wrong but nothing faults
          tma_load_4d(base + dh * (kN * 128) + c * 16 * 128, &kvmap, dh * 64, rec.h,
                      (tok_tile + c * 16) % p.ps, (bad ? 0 : page) * 2 + which, full, pol_kv);
          if (bad && dh == 0 && which == 0) flag(p.status, MI_STATUS_BAD_PAGE);
        }
        return true;
      };
      // K runs one tile ahead of V: K0, K1, V0, K2, V1, ..., V(n-1)
      int pg_prev = -1;
      for (int j = 0; j < rec.n_tiles && ok; ++j, ++gt) {
        if (j > 0 && (j & 3) == 0) {  // next window of page ids
          pw = pwn;
          pwn = load_win((j >> 2) + 1);
        }
        const int pg = __shfl_sync(0xffffffffu, pw, ((j & 3) << 3) + min(lane / DH, 7));
        if (!issue(j, gt, 0, pg)) ok = false;
        if (ok && j + 1 == rec.n_tiles && lane == 0 && p.ctr)
          k_ahead = static_cast<int>(atomicAdd(p.ctr, 1u));  // used after the V tiles below
        if (ok && j > 0 && !issue(j - 1, gt - 1, 1, pg_prev)) ok = false;
        pg_prev = pg;
      }
      if (ok && !issue(rec.n_tiles - 1, gt - 1, 1, pg_prev)) ok = false;
    }
    // no copy may be in flight when the CTA retires
    for (int t = max(0, qc - L::NQ); t < qc; ++t)
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&q_full[t % L::NQ], (t / L::NQ) & 1)))
        ok = false;
    for (int t = max(0, gt - L::NK); t < gt; ++t)
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&k_full[t % L::NK], (t / L::NK) & 1)))
        ok = false;
    for (int t = max(0, gt - L::NV); t < gt; ++t)
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&v_full[t % L::NV], (t / L::NV) & 1)))
        ok = false;
  } else if (warp == 1) {
    // ============================ MMA issuer ================================
    if (lane == 0) {
      const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      const uint32_t idesc_qk = umma_idesc(fmt, false, kN, kM);
      const uint32_t idesc_pv = umma_idesc(fmt, true, D, kM);
      const uint32_t tmem_p = tmem + L::P_COL;
      auto issue_qk = [&](int t, int qb) {  // S = Q K^T of global tile t (stage t & 1), Q buffer qb
        const uint32_t q_addr = smem_u32(smem + L::Q_OFF + qb * L::Q_BYTES);
        const uint32_t k_addr = smem_u32(smem + L::K_OFF + (t % L::NK) * L::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kM * 128) + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * (kN * 128) + (kk & 3) * 32;
          umma(tmem_s, umma_desc(q_addr + off, 16, 1024), umma_desc(k_addr + koff, 16, 1024),
               idesc_qk, kk > 0);
        }
        umma_commit(s_full);
        umma_commit(&k_empty[t % L::NK]);
      };
      // Items come in order; the next item with keys is looked up ahead so
      // its first QK^T can run under the softmax of this item's last tile.
      int it = 0, gt = 0, qc = 0, oc = 0;
      auto next_item = [&](PfItem &r) -> bool {  // the next record with keys; false at the end
        for (;;) {
          const int slot = it & 1;
          if (!mbar_wait_bounded(&it_full[slot], (it >> 1) & 1)) { ok = false; return false; }
          r = items[slot];
          mbar_arrive(&it_empty[slot]);  // the record is copied
          ++it;
          if (r.b < 0) return false;
          if (r.n_tiles > 0) return true;
        }
      };
      PfItem cur, nxt;
      bool have = next_item(cur), have_next = false;
      if (have) {  // first QK^T
        if (!mbar_wait_bounded(&q_full[0], 0) || !mbar_wait_bounded(&k_full[0], 0)) ok = false;
        if (ok) {
          tc_fence_after();
          issue_qk(0, 0);
          if (cur.n_tiles == 1) umma_commit(&q_empty[0]);
        }
      }
      int last_gt = -1;
      while (have && ok) {
        const int ob = oc & 1;
        const uint32_t tmem_o = tmem + L::O_COL + ob * L::OB_STRIDE;
        for (int j = 0; j < cur.n_tiles && ok; ++j, ++gt) {
          // look ahead: QK^T of the next tile (this item's, or the next item's first)
          bool ahead = j + 1 < cur.n_tiles;
          bool cross = false;
          if (!ahead) {
            have_next = next_item(nxt);
            ahead = cross = have_next;
          }
          if (ahead) {
            const int qn = cross ? qc + 1 : qc;  // the item the next tile belongs to
            if (!mbar_wait_bounded(s_free, gt & 1) ||
                (cross && !mbar_wait_bounded(&q_full[qn % L::NQ], (qn / L::NQ) & 1)) ||
                !mbar_wait_bounded(&k_full[(gt + 1) % L::NK], ((gt + 1) / L::NK) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_qk(gt + 1, qn % L::NQ);
            // the last QK^T of its item frees its Q buffer for a later item
            const bool last_qk = cross ? nxt.n_tiles == 1 : j + 2 == cur.n_tiles;
            if (last_qk) umma_commit(&q_empty[qn % L::NQ]);
          }
          if (!mbar_wait_bounded(p_full, gt & 1) ||
              !mbar_wait_bounded(&v_full[gt % L::NV], (gt / L::NV) & 1)) {
            ok = false;
            break;
          }
          if (j == 0 && oc >= 2 && !mbar_wait_bounded(&o_free[ob], ((oc >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + L::V_OFF + (gt % L::NV) * L::V_BYTES);
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk) {
            // P from TMEM (16 keys = 8 columns per step); V: MN-major, 64-wide d
            // blocks kN*128 bytes apart, 8-token groups 1 KB apart
            umma_ts(tmem_o, tmem_p + kk * 8, umma_desc(v_addr + kk * 16 * 128, kN * 128, 1024),
                    idesc_pv, (j > 0 || kk > 0));
          }
          umma_commit(&v_empty[gt % L::NV]);
          umma_commit(o_done);
          if (j + 1 == cur.n_tiles) umma_commit(&o_full[ob]);
          last_gt = gt;
        }
        ++qc;
        ++oc;
        have = have_next;
        cur = nxt;
        have_next = false;
      }
      // the last products must land before TMEM is freed
      if (last_gt >= 0 && !mbar_wait_bounded(o_done, last_gt & 1)) ok = false;
    }
    __syncwarp();
  } else if (warp < 10) {
    // ======================== softmax (warps 2..9) ===========================
    // Two halves of four warps each: the half sg owns S columns
    // [64 sg, 64 sg + 64) (and so the P block sg) and O columns
    // [D/2 sg, D/2 sg + D/2); thread = TMEM lane = packed query row in both.
    // Per tile the halves swap their row maxima (xch) through shared memory
    // behind a bounded mbarrier wait. At an item's end they leave its row
    // sums, row max and output record for the epilogue warps (l_ready) and go
    // on with the next item while O is read out.
    constexpr int SC = kN / 2, OC = D / 2;
    const int sg = (warp - 2) >> 2;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // packed row == TMEM lane
    const int t = r / g, jh = r % g;
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t tmem_p = tmem + L::P_COL + lane_base + sg * (SC / 2);  // this half's P columns
    float *xmax = reinterpret_cast<float *>(smem + L::XCH_OFF);  // [tile & 1][half][row]
    float *lsum = reinterpret_cast<float *>(smem + L::LSUM_OFF);  // [ob][half][row]
    float *mfin = reinterpret_cast<float *>(smem + L::MFIN_OFF);  // [ob][row]
    int4 *erec = reinterpret_cast<int4 *>(smem + L::EREC_OFF);    // [ob]
    int gt = 0, oc = 0;
    // hand buffer ob's record to the epilogue warps once they have finished
    // with that buffer's previous item (its o_free)
    auto hand_off = [&](int ob, int4 er, float l, float m) -> bool {
      if (oc >= 2 &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(&o_free[ob], ((oc >> 1) - 1) & 1)))
        return false;
      lsum[(ob * 2 + sg) * kM + r] = l;
      if (sg == 0) mfin[ob * kM + r] = m;
      if (warp == 2 && lane == 0) erec[ob] = er;
      __syncwarp();
      if (lane == 0) mbar_arrive(&l_ready[ob]);
      return true;
    };
    for (int it = 0; ok; ++it) {
      const int slot = it & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&it_full[slot], (it >> 1) & 1))) {
        ok = false;
        break;
      }
      const PfItem rec = items[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&it_empty[slot]);
      if (rec.b < 0) {  // no more items: an end record for the epilogue warps
        if (!hand_off(oc & 1, make_int4(-1, 0, 0, 0), 0.f, 0.f)) ok = false;
        break;
      }
      const int rows_tok = min(tq, rec.lq - rec.t0);
      const bool row_ok = r < m_used && t < rows_tok;
      const int64_t orow = static_cast<int64_t>(rec.q_start + rec.t0 + t) * p.hq + rec.h * g + jh;
      if (rec.n_tiles == 0) {  // no visible key: zeros, lse = -inf
        if (row_ok) {
          T *o = static_cast<T *>(p.out) + orow * D + sg * OC;
          for (int i = 0; i < OC; ++i) o[i] = Elt<T>::from(0.f);
          if (p.lse && sg == 0) p.lse[orow] = -INFINITY;
        }
        continue;
      }
      int lim = p.causal ? rec.lk - rec.lq + rec.t0 + t + 1 : rec.lk;
      lim = min(lim, rec.lk);
      if (!row_ok) lim = 0;
      const int ob = oc & 1;
      const uint32_t tmem_o = tmem + L::O_COL + ob * L::OB_STRIDE + sg * OC;
      float m = -INFINITY, l = 0.f;  // l: this half's share of the row sum
      for (int j = 0; j < rec.n_tiles; ++j, ++gt) {
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(s_full, gt & 1))) { ok = false; break; }
        tc_fence_after();
        float sv[SC];
#pragma unroll
        for (int c = 0; c < SC / 32; ++c)
          tmem_ld32(tmem_s + sg * SC + lane_base + c * 32, sv + c * 32);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);
        // raw scores; the scale is folded into the exponent's FMA below.
        // Keys past a row's limit count as -inf; only warps with such a row
        // in this tile pay for the mask.
        const int kbase = j * kN + sg * SC;
        if (__any_sync(0xffffffffu, kbase + SC > lim)) {
#pragma unroll
          for (int c = 0; c < SC; ++c) sv[c] = (kbase + c < lim) ? sv[c] : -INFINITY;
        }
        float mt = -INFINITY;
#pragma unroll
        for (int c = 0; c < SC; ++c) mt = fmaxf(mt, sv[c]);
        mt *= p.scale_log2;  // scale_log2 > 0: the max commutes with it
        // row max over both halves
        float *xm = xmax + (gt & 1) * 2 * kM;
        xm[sg * kM + r] = mt;
        __syncwarp();
        if (lane == 0) mbar_arrive(xch);
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(xch, gt & 1))) { ok = false; break; }
        mt = fmaxf(mt, xm[(sg ^ 1) * kM + r]);
        // keep the old max unless this tile's exceeds it by > kRescaleLog2
        // (both halves see the same maxima, so they take the same decision)
        const float m_new = (mt > m + kRescaleLog2 || m == -INFINITY) ? fmaxf(m, mt) : m;
        const float ms = m_new == -INFINITY ? 0.f : m_new;
        const float corr = m == m_new ? 1.f : fast_exp2(m - ms);
        float sum = 0.f;
#pragma unroll
        for (int c = 0; c < SC; ++c) {
          sv[c] = fast_exp2(fmaf(sv[c], p.scale_log2, -ms));
          sum += sv[c];
        }
        l = l * corr + sum;
        m = m_new;
        // the previous tile's P V must be done: P is rewritten, O rescaled
        if (gt > 0) {
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(o_done, (gt - 1) & 1))) { ok = false; break; }
          tc_fence_after();
        }
        {  // P row: SC keys as 16-bit pairs into this half's TMEM columns
          float pk[SC / 2];
#pragma unroll
          for (int c = 0; c < SC / 2; ++c) pk[c] = __uint_as_float(Pack2<T>::run(sv[2 * c], sv[2 * c + 1]));
          tmem_st32(tmem_p, pk);
        }
        if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
          for (int c = 0; c < OC / 32; ++c) {
            float ov[32];
            tmem_ld32(tmem_o + lane_base + c * 32, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= corr;
            tmem_st32(tmem_o + lane_base + c * 32, ov);
          }
        }
        tmem_wait_st();  // P (and a rescaled O) are in TMEM before the MMA is told
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
      }
      if (!ok) break;
      if (!hand_off(ob, make_int4(rec.q_start + rec.t0, rec.h, rows_tok, 0), l, m)) {
        ok = false;
        break;
      }
      ++oc;
    }
  } else {
    // ======================= epilogue (warps 10..13) =========================
    // Thread = TMEM lane = packed query row, all head_dim columns. Per item
    // (in the order the softmax warps finish them, O buffers alternating):
    // wait for the item's last P V (o_full) and its row sums (l_ready),
    // normalise O, store it, release the O buffer (o_free).
    const int qd = warp & 3;  // the TMEM lane quarter this warp may access
    const int r = qd * 32 + lane;
    const int t = r / g, jh = r % g;
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const float *lsum = reinterpret_cast<const float *>(smem + L::LSUM_OFF);
    const float *mfin = reinterpret_cast<const float *>(smem + L::MFIN_OFF);
    const int4 *erec = reinterpret_cast<const int4 *>(smem + L::EREC_OFF);
    for (int oc = 0; ok; ++oc) {
      const int ob = oc & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&l_ready[ob], (oc >> 1) & 1))) {
        ok = false;
        break;
      }
      const int4 er = erec[ob];  // token base, KV head, query tokens; x < 0: the end
      if (er.x < 0) break;
      const float l = lsum[(ob * 2) * kM + r] + lsum[(ob * 2 + 1) * kM + r];
      const float m = mfin[ob * kM + r];
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&o_full[ob], (oc >> 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool row_ok = r < m_used && t < er.z;
      const int64_t orow = static_cast<int64_t>(er.x + t) * p.hq + er.y * g + jh;
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T *o = static_cast<T *>(p.out) + orow * D;
      const uint32_t tmem_o = tmem + L::O_COL + ob * L::OB_STRIDE;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float ov[32];
        tmem_ld32(tmem_o + lane_base + c * 32, ov);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = Pack2<T>::run(ov[i] * inv, ov[i + 1] * inv);
            w.y = Pack2<T>::run(ov[i + 2] * inv, ov[i + 3] * inv);
            w.z = Pack2<T>::run(ov[i + 4] * inv, ov[i + 5] * inv);
            w.w = Pack2<T>::run(ov[i + 6] * inv, ov[i + 7] * inv);
            *reinterpret_cast<uint4 *>(o + c * 32 + i) = w;
          }
        }
      }
      if (row_ok && p.lse) p.lse[orow] = l > 0.f ? (m + __log2f(l)) * kLn2 : -INFINITY;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[ob]);  // O buffer ob may be overwritten
    }
  }
  if (!ok && lane == 0) flag(p.status, MI_STATUS_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(L::TMEM_COLS)
                 : "memory");
  }
  // the last CTA out resets the shared item counters for the next launch
  if (threadIdx.x == 0 && p.ctr) {
    __threadfence();
    if (atomicAdd(p.ctr + 1, 1u) + 1u == gridDim.x) {
      p.ctr[0] = 0u;
      p.ctr[1] = 0u;
      __threadfence();
    }
  }
}

template <typename T, int D>
int launch_t(const PrefillParams &p, int dtype, cudaStream_t s) {
  using L = PfLayout<D>;
  CUtensorMap qmap, kvmap;
  const int tq = kM / p.group;
  if (!rows_tensor_map(p.q, p.total_q, p.hq, D, p.qsn, p.qsh, p.group, tq, dtype, &qmap))
    return -1;
  if (!pool_tensor_map(p.kv, p.num_pages, p.ps, p.hkv, D, dtype, &kvmap)) return -1;
  static std::atomic<unsigned long long> attr_set{0};
  if (smem_limit_once(attr_set, prefill_tc_kernel<T, D>, L::SMEM) != cudaSuccess)
    return check_launch("prefill_tc_kernel smem attribute");
  // persistent: one CTA per SM, or fewer when there are fewer work items
  // (an upper bound on the items: (sum ceil(L_b / tq)) * hkv <= (total/tq + batch) * hkv)
  const int64_t items = (static_cast<int64_t>(p.total_q) / tq + p.batch) * p.hkv;
  const int grid = static_cast<int>(std::min<int64_t>(items, num_sms()));
  prefill_tc_kernel<T, D><<<grid, kThreadsP, L::SMEM, s>>>(qmap, kvmap, p);
  return check_launch("prefill_tc_kernel");
}

}  // namespace

int launch_prefill_tc(const PrefillParams &p, int dtype, cudaStream_t s) {
  if (!(dtype == MI_DTYPE_BF16 || dtype == MI_DTYPE_F16)) return -1;
  if (!(p.d == 64 || p.d == 128)) return -1;
  if (p.group > kM || p.ps % 16 != 0 || p.ps > 256 || p.batch > kMaxBatchTc) return -1;
  if (p.hkv > 65535 || p.num_pages * 2 > (1LL << 31)) return -1;
  if (!(p.scale_log2 > 0.f)) return -1;  // the softmax takes the row max before scaling
  if (static_cast<int64_t>(p.total_q) + kM > (1LL << 31)) return -1;
  if (dtype == MI_DTYPE_BF16)
    return p.d == 128 ? launch_t<__nv_bfloat16, 128>(p, dtype, s)
                      : launch_t<__nv_bfloat16, 64>(p, dtype, s);
  return p.d == 128 ? launch_t<__half, 128>(p, dtype, s) : launch_t<__half, 64>(p, dtype, s);
}

}  // namespace mi
