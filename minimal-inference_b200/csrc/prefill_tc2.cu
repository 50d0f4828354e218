// Kernel (3), two query tiles per work item: paged prefill attention on
// tcgen05 / TMEM, the softmax of one query tile running under the other's
// tensor-core products.
//
// Replaces the FlashInfer paged prefill the reference runs
// (scheduler.py:530-534, :704-716, model.py:235) for bf16 / fp16, head_dim
// 64 / 128, page_size a multiple of 16 (the generic kernel in prefill.cu
// takes every other shape). A work item is
// (request, KV head, 256 packed query rows): two query tiles A and B of 128
// rows, a row being a (query token, query head of the GQA group) pair, so a
// tile holds Tq = 128 / group tokens and every K/V tile brought in serves
// 2 Tq tokens of the whole group (half the K/V loads per query row of a
// one-tile item, and half the items). The grid is persistent, one CTA per
// SM, items taken from a counter in the workspace (each request's heaviest
// query tiles first). 14 warps:
//   warp 0      producer: TMA loads of the two Q tiles (3-D map over q) and
//               of 128-token K/V tiles straight from the pages (4-D pool map,
//               16-token boxes), two K and two V stages, 128-byte swizzle;
//   warp 1      MMA issuer (one thread). Per K/V tile j the tensor pipe runs
//               P_A V_j, S_A(j+1) = Q_A K_{j+1}^T, P_B V_j, S_B(j+1): while
//               one tile's softmax warps work on S, the pipe works for the
//               other tile;
//   warps 2-5   softmax of tile A, warps 6-9 softmax of tile B: thread = TMEM
//               lane = packed row, the whole 128-key row of S in one pass
//               over TMEM against the running max (in an item's first tile,
//               the max of its first 32 keys): exp2, row sum, 16-bit P
//               written over S columns already read, chunk by chunk; from
//               the first chunk with a key more than 2^8 above that max the
//               tile takes two passes (row max first) against a new max,
//               the P already written is rebased, and O is rescaled in TMEM
//               only then;
//   warps 10-13 epilogue: normalise a finished item's O_A and O_B and store
//               them, releasing each O buffer as soon as it is read.
// An item's last tile is a half tile when at most 64 of its keys are visible
// to the item's rows (causal diagonal, ragged end): its products cover those
// 64 keys only (QK^T with N = 64, P V over 4 key steps).
// TMEM (512 columns): S_A [0,128), S_B [128,256) with P_A / P_B in their
// first 64 columns; O_A and O_B (head_dim columns each) from column 256.
// Every wait is bounded; TMEM is freed on every path.
#include <algorithm>
#include <type_traits>

#include "prefill.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace mi {
namespace {

constexpr int kM = 128;         // packed query rows per tile
constexpr int kN = 128;         // KV tokens per tile
constexpr int kThreads2 = 448;  // producer, MMA, 2 x 4 softmax warps, 4 epilogue warps
constexpr int kMaxBatch2 = 1024;
constexpr int kSortBatch = 128;  // requests ordered by length up to this batch

template <int D> struct Pf2Layout {
  static constexpr int DH = D / 64;                 // 64-wide blocks of head_dim
  static constexpr int Q_BYTES = DH * kM * 128;     // one query tile, [dh][row][64]
  static constexpr int K_BYTES = DH * kN * 128;     // [dh][token][64]
  static constexpr int V_BYTES = K_BYTES;
  static constexpr int NK = 2, NV = 2;              // K and V stages
  static constexpr int Q_OFF = 0;                   // tiles A and B
  static constexpr int K_OFF = Q_OFF + 2 * Q_BYTES;
  static constexpr int V_OFF = K_OFF + NK * K_BYTES;
  static constexpr int BAR_OFF = V_OFF + NV * V_BYTES;  // 35 mbarriers + the TMEM base
  static constexpr int ITEM_OFF = BAR_OFF + 320;       // 2 work-item records
  // hand-off to the epilogue, per slot (item parity) and tile: row sums,
  // row maxima; per slot the output record
  static constexpr int LSUM_OFF = ITEM_OFF + 2 * 48;
  static constexpr int MFIN_OFF = LSUM_OFF + 2 * 2 * kM * 4;
  static constexpr int EREC_OFF = MFIN_OFF + 2 * 2 * kM * 4;
  static constexpr int META_OFF = EREC_OFF + 2 * 16;
  // item prefix, qo_indptr, kv_indptr [batch+1], kv_len [batch] and the
  // request order [batch]
  static constexpr int META_INTS = 5 * (kMaxBatch2 + 1);
  static constexpr int SMEM = META_OFF + META_INTS * 4 + 1024;
  static constexpr int S_COL = 0;      // S_A at 0, S_B at kN (P over the first kN / 2)
  static constexpr int O_COL = 2 * kN; // O_A, O_B: D columns each
  static constexpr int TMEM_COLS = 512;
};

struct __align__(16) Pf2Item {
  int b, h, t0, n_tiles;  // b < 0: no more items
  int q_start, lq, lk, page_base;
  int last_keys;          // keys of the last tile visible to some row of the item
  int pad[3];
};

template <typename T, int D>
// 14 warps: four of them share one SM sub-partition's 16 K registers, so at
// most 128 registers per thread
__global__ void __launch_bounds__(kThreads2, 1)
    prefill_tc2_kernel(const __grid_constant__ CUtensorMap qmap,
                       const __grid_constant__ CUtensorMap kvmap, const PrefillParams p) {
  using L = Pf2Layout<D>;
  constexpr int DH = L::DH;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  uint64_t *it_full = bars + 0, *it_empty = bars + 2;
  uint64_t *q_full = bars + 4, *q_empty = bars + 6;       // [tile]
  uint64_t *k_full = bars + 8, *k_empty = bars + 10;      // [stage]
  uint64_t *v_full = bars + 12, *v_empty = bars + 14;     // [stage]
  uint64_t *s_full = bars + 16, *p_full = bars + 18;      // [tile]
  uint64_t *pv_done = bars + 20, *o_full = bars + 22;     // [tile]
  uint64_t *o_free = bars + 24;                           // [tile]
  uint64_t *l_ready = bars + 26;                          // [slot * 2 + tile]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 30);
  uint64_t *drain = bars + 32;   // one final commit: every product has landed
  uint64_t *h_free = bars + 33;  // [slot * 2 + tile]: the epilogue has read the slot's hand-off
  Pf2Item *items = reinterpret_cast<Pf2Item *>(smem + L::ITEM_OFF);
  int *tiles_pre = reinterpret_cast<int *>(smem + L::META_OFF);
  int *s_qo = tiles_pre + (kMaxBatch2 + 1);
  int *s_ip = s_qo + (kMaxBatch2 + 1);
  int *s_lk = s_ip + (kMaxBatch2 + 1);
  int *s_order = s_lk + (kMaxBatch2 + 1);  // work-item order of the requests

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = p.group;
  const int tq = kM / g;        // query tokens per tile
  const int m_used = tq * g;    // packed rows in use per tile
  const int tq2 = 2 * tq;       // query tokens per item

  // ---- once per CTA: item prefix over requests, barriers, TMEM ------------
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
  __syncthreads();
  // Requests in decreasing query length (ties by index), so the queue ends
  // with the shortest requests' light items and the CTAs finish together
  // (rank by counting: batch^2 / blockDim comparisons per thread, so only up
  // to kSortBatch requests; larger batches keep their order).
  for (int i = threadIdx.x; i < p.batch; i += blockDim.x) {
    int rank = i;
    if (p.batch <= kSortBatch) {
      const int li = s_qo[i + 1] - s_qo[i];
      rank = 0;
      for (int j = 0; j < p.batch; ++j) {
        const int lj = s_qo[j + 1] - s_qo[j];
        rank += (lj > li || (lj == li && j < i)) ? 1 : 0;
      }
    }
    s_order[rank] = i;
  }
  __syncthreads();
  if (warp == 0) {  // tiles_pre[i] = sum over the first i requests in s_order of ceil(qo_len / (2 Tq))
    int carry = 0;
    if (lane == 0) tiles_pre[0] = 0;
    for (int base = 0; base < p.batch; base += 32) {
      const int bb = base + lane;
      const int rb = bb < p.batch ? s_order[bb] : 0;
      int x = bb < p.batch ? cdiv(max(0, s_qo[rb + 1] - s_qo[rb]), tq2) : 0;
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
      for (int i = 0; i < 2; ++i) {
        mbar_init(&it_full[i], 1);
        mbar_init(&it_empty[i], 9);   // the MMA thread and the 8 softmax warps
        mbar_init(&q_full[i], 1);
        mbar_init(&q_empty[i], 1);
        mbar_init(&k_full[i], 1);
        mbar_init(&k_empty[i], 1);
        mbar_init(&v_full[i], 1);
        mbar_init(&v_empty[i], 1);
        mbar_init(&s_full[i], 1);
        mbar_init(&p_full[i], 4);     // the tile's 4 softmax warps
        mbar_init(&pv_done[i], 1);
        mbar_init(&o_full[i], 1);
        mbar_init(&o_free[i], 4);     // the 4 epilogue warps
        mbar_init(&l_ready[2 * i], 4);
        mbar_init(&l_ready[2 * i + 1], 4);
        mbar_init(&h_free[2 * i], 4);
        mbar_init(&h_free[2 * i + 1], 4);
      }
      mbar_init(drain, 1);
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
  const int n_items = tiles_pre[p.batch] * p.hkv;
  bool ok = true;

  if (warp == 0) {
    // ============================ producer ==================================
    // a Q tile is read by one work item; a request's K/V tiles by every
    // query chunk of the request: K/V are the lines worth keeping in L2
    const uint64_t pol_q = evict_first_policy(), pol_kv = evict_last_policy();
    int gt = 0, qc = 0;
    int k_ahead = -1;  // lane 0: the next item's index, taken while this item's last V tiles go out
    for (int it = 0; ok; ++it) {
      int k = 0;
      if (lane == 0) {
        k = k_ahead >= 0 ? k_ahead
                         : (p.ctr ? static_cast<int>(atomicAdd(p.ctr, 1u)) : blockIdx.x + it * gridDim.x);
        k_ahead = -1;
      }
      k = __shfl_sync(0xffffffffu, k, 0);
      Pf2Item rec{-1, 0, 0, 0, 0, 0, 0, 0, 0, {0, 0, 0}};
      if (k < n_items) {
        int lo = 0, hi = p.batch - 1;  // last position with tiles_pre[pos] * hkv <= k
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (tiles_pre[mid] * p.hkv <= k) lo = mid; else hi = mid - 1;
        }
        const int b = s_order[lo], ntq = tiles_pre[lo + 1] - tiles_pre[lo];
        const int rem = k - tiles_pre[lo] * p.hkv;
        rec.b = b;
        // the request's query chunks heaviest (last) first, all KV heads of
        // a chunk together
        rec.h = rem % p.hkv;
        rec.t0 = (ntq - 1 - rem / p.hkv) * tq2;
        rec.q_start = s_qo[b];
        rec.lq = s_qo[b + 1] - rec.q_start;
        rec.lk = s_lk[b];
        rec.page_base = s_ip[b];
        const int rows_tok = min(tq2, rec.lq - rec.t0);
        const int lim_tok =
            p.causal ? min(rec.lk, rec.lk - rec.lq + rec.t0 + rows_tok) : rec.lk;
        rec.n_tiles = lim_tok > 0 ? cdiv(lim_tok, kN) : 0;
        rec.last_keys = lim_tok - (rec.n_tiles - 1) * kN;
      }
      const int slot = it & 1;
      if (it >= 2 &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(&it_empty[slot], ((it >> 1) - 1) & 1))) {
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
      // and the next window in registers
      const int nchunk = rec.n_tiles * 8;
      auto load_win = [&](int w) -> int {
        const int c = w * 32 + lane;
        return c < nchunk && c * 16 < rec.lk ? p.indices[rec.page_base + (c * 16) / p.ps] : -1;
      };
      int pw = load_win(0), pwn = load_win(1);
      // the two Q tiles, each once the previous item's last QK^T of that
      // tile is done
      for (int x = 0; x < 2 && ok; ++x) {
        if (qc >= 1 && !__all_sync(0xffffffffu, mbar_wait_bounded(&q_empty[x], (qc - 1) & 1))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&q_full[x], DH * m_used * 128);
          for (int dh = 0; dh < DH; ++dh)
            tma_load_3d(smem + L::Q_OFF + x * L::Q_BYTES + dh * kM * 128, &qmap, dh * 64,
                        rec.h * g, rec.q_start + rec.t0 + x * tq, &q_full[x], pol_q);
        }
      }
      if (!ok) break;
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
        // 16-token chunks up to the item's last visible key. Past it no row
        // sees a key: every warp masks those S columns (P = 0), and a half
        // tile's products do not reach them.
        const int nvc = min(8, cdiv((j + 1 == rec.n_tiles ? rec.last_keys : kN), 16));
        unsigned char *base = smem + (which ? L::V_OFF + st * L::V_BYTES : L::K_OFF + st * L::K_BYTES);
        if (which == 1 && gtile < L::NV && nvc < 8) {
          // V chunks not loaded are multiplied by P = 0; on a stage's first
          // use they hold whatever shared memory held, so zero them (later
          // uses keep an earlier tile's finite values there)
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
      // in the order the tensor core uses them, which is also the order
      // their stages free up: K0, V0, K1, V1, ..., K(n-1), V(n-1)
      int pg_prev = -1;
      for (int j = 0; j < rec.n_tiles && ok; ++j, ++gt) {
        if (j > 0 && !issue(j - 1, gt - 1, 1, pg_prev)) ok = false;
        if (j > 0 && (j & 3) == 0) {  // next window of page ids
          pw = pwn;
          pwn = load_win((j >> 2) + 1);
        }
        const int pg = __shfl_sync(0xffffffffu, pw, ((j & 3) << 3) + min(lane / DH, 7));
        if (ok && !issue(j, gt, 0, pg)) ok = false;
        if (ok && j + 1 == rec.n_tiles && lane == 0 && p.ctr)
          k_ahead = static_cast<int>(atomicAdd(p.ctr, 1u));  // used after the V tile below
        pg_prev = pg;
      }
      if (ok && !issue(rec.n_tiles - 1, gt - 1, 1, pg_prev)) ok = false;
    }
    // no copy may be in flight when the CTA retires
    if (qc >= 1)
      for (int x = 0; x < 2; ++x)
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&q_full[x], (qc - 1) & 1))) ok = false;
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
      const uint32_t idesc_qk_half = umma_idesc(fmt, false, kN / 2, kM);
      const uint32_t idesc_pv = umma_idesc(fmt, true, D, kM);
      // tile B of the current item lies past its request's end (the request
      // ends inside tile A): its products are not issued, its commits are
      bool skip_b = false;
      // S_x = Q_x K^T of global tile t (K stage t % NK); a half tile (the
      // item's last, with at most kN / 2 visible keys) computes its first
      // kN / 2 columns only
      // descriptors of the stage bases; a descriptor's start field is the
      // address / 16 (shared memory < 256 KB), so an offset adds offset / 16
      const uint64_t qdesc0 = umma_desc(smem_u32(smem + L::Q_OFF), 16, 1024);
      const uint64_t kdesc0 = umma_desc(smem_u32(smem + L::K_OFF), 16, 1024);
      const uint64_t vdesc0 = umma_desc(smem_u32(smem + L::V_OFF), kN * 128, 1024);
      auto issue_qk = [&](int t, int x, bool half) {
        const uint64_t qd = qdesc0 + ((x * L::Q_BYTES) >> 4);
        const uint64_t kd = kdesc0 + (((t % L::NK) * L::K_BYTES) >> 4);
        const uint32_t id = half ? idesc_qk_half : idesc_qk;
        const uint32_t d_col = tmem + L::S_COL + x * kN;
#pragma unroll
        for (int kk = 0; kk < D / 16 && !(x == 1 && skip_b); ++kk) {
          const uint32_t off = (kk >> 2) * (kM * 128) + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * (kN * 128) + (kk & 3) * 32;
          umma(d_col, qd + (off >> 4), kd + (koff >> 4), id, kk > 0);
        }
        umma_commit(&s_full[x]);
      };
      // O_x (+)= P_x V of global tile t (V stage t % NV); P from TMEM (16
      // keys = 8 columns per step), V MN-major: 64-wide d blocks kN*128
      // bytes apart, 8-token groups 1 KB apart; a half tile's first kN / 2
      // keys only
      auto issue_pv = [&](int t, int x, bool acc, bool half) {
        const uint64_t vd = vdesc0 + (((t % L::NV) * L::V_BYTES) >> 4);
        const uint32_t o_col = tmem + L::O_COL + x * D, p_col = tmem + L::S_COL + x * kN;
#pragma unroll
        for (int kk = 0; kk < kN / 16 && !(x == 1 && skip_b); ++kk)
          if (!half || kk < kN / 32)
            umma_ts(o_col, p_col + kk * 8, vd + ((kk * 16 * 128) >> 4), idesc_pv, acc || kk > 0);
        umma_commit(&pv_done[x]);
      };
      int gt = 0, oc = 0;
      bool issued = false;  // any product issued (the drain below then waits for them)
      for (int it = 0; ok; ++it) {
        const int slot = it & 1;
        if (!mbar_wait_bounded(&it_full[slot], (it >> 1) & 1)) { ok = false; break; }
        const Pf2Item rec = items[slot];
        mbar_arrive(&it_empty[slot]);  // the record is copied
        if (rec.b < 0) break;
        const int n = rec.n_tiles;
        if (n == 0) continue;
        const bool half_last = rec.last_keys <= kN / 2;  // the last tile is a half tile
        skip_b = rec.lq - rec.t0 <= tq;
        // first products of the item: S_A(0), S_B(0), each once the previous
        // item's last P_x V has completed. S_x is written over P_x, which
        // that product reads from TMEM, and products into different TMEM
        // accumulators are not ordered by their issue order.
        for (int x = 0; x < 2 && ok; ++x) {
          if (!mbar_wait_bounded(&q_full[x], oc & 1) ||
              (x == 0 && !mbar_wait_bounded(&k_full[gt % L::NK], (gt / L::NK) & 1)) ||
              (gt >= 1 && !mbar_wait_bounded(&pv_done[x], (gt - 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_qk(gt, x, n == 1 && half_last);
          issued = true;
          if (n == 1) umma_commit(&q_empty[x]);
        }
        if (!ok) break;
        umma_commit(&k_empty[gt % L::NK]);
        for (int j = 0; j < n && ok; ++j) {
          const int t = gt + j;
          for (int x = 0; x < 2; ++x) {
            // O_x += P_x V_t once the tile's softmax warps have written P_x
            // (and the epilogue has read the previous item's O_x)
            if (!mbar_wait_bounded(&p_full[x], t & 1) ||
                (x == 0 && !mbar_wait_bounded(&v_full[t % L::NV], (t / L::NV) & 1)) ||
                (j == 0 && oc >= 1 && !mbar_wait_bounded(&o_free[x], (oc - 1) & 1))) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, x, j > 0, j + 1 == n && half_last);
            if (x == 1) umma_commit(&v_empty[t % L::NV]);
            if (j + 1 == n) umma_commit(&o_full[x]);
            if (j + 1 < n) {
              // S_x of the next tile overwrites P_x: its P V must be done
              if ((x == 0 && !mbar_wait_bounded(&k_full[(t + 1) % L::NK], ((t + 1) / L::NK) & 1)) ||
                  !mbar_wait_bounded(&pv_done[x], t & 1)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_qk(t + 1, x, j + 2 == n && half_last);
              if (x == 1) umma_commit(&k_empty[(t + 1) % L::NK]);
              if (j + 2 == n) umma_commit(&q_empty[x]);  // the item's last QK^T of tile x
            }
          }
        }
        gt += n;
        ++oc;
      }
      // every product must land before TMEM is freed: a commit tracks all
      // of this thread's earlier tensor-core operations
      if (issued) {
        umma_commit(drain);
        if (!mbar_wait_bounded(drain, 0)) ok = false;
      }
    }
    __syncwarp();
  } else if (warp < 10) {
    // ======================== softmax (warps 2..9) ===========================
    const int x = (warp - 2) >> 2;  // query tile: 0 = A, 1 = B
    const int qd = warp & 3;        // the TMEM lane quarter this warp may access
    const int r = qd * 32 + lane;   // packed row == TMEM lane
    const int t = r / g, jh = r % g;
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t tmem_s = tmem + L::S_COL + x * kN + lane_base;
    const uint32_t tmem_o = tmem + L::O_COL + x * D + lane_base;
    float *lsum = reinterpret_cast<float *>(smem + L::LSUM_OFF);  // [slot][tile][row]
    float *mfin = reinterpret_cast<float *>(smem + L::MFIN_OFF);  // [slot][tile][row]
    int4 *erec = reinterpret_cast<int4 *>(smem + L::EREC_OFF);    // [slot]
    int gt = 0, oc = 0;
    // hand item oc's row sums / maxima (and, from tile A, its output record)
    // to the epilogue once it has read the slot's previous contents (item
    // oc - 2; a barrier per slot, so its parity names that item alone)
    auto hand_off = [&](int4 er, float l, float m) -> bool {
      const int slot = oc & 1;
      if (oc >= 2 && !__all_sync(0xffffffffu,
                                 mbar_wait_bounded(&h_free[slot * 2 + x], ((oc >> 1) - 1) & 1)))
        return false;
      lsum[(slot * 2 + x) * kM + r] = l;
      mfin[(slot * 2 + x) * kM + r] = m;
      if (x == 0 && warp == 2 && lane == 0) erec[slot] = er;
      __syncwarp();
      if (lane == 0) mbar_arrive(&l_ready[slot * 2 + x]);
      return true;
    };
    for (int it = 0; ok; ++it) {
      const int slot = it & 1;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&it_full[slot], (it >> 1) & 1))) {
        ok = false;
        break;
      }
      const Pf2Item rec = items[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&it_empty[slot]);
      if (rec.b < 0) {  // no more items: tile A tells the epilogue warps
        if (x == 0 && !hand_off(make_int4(-1, 0, 0, 0), 0.f, 0.f)) ok = false;
        break;
      }
      const int rows_tok = max(0, min(tq, rec.lq - rec.t0 - x * tq));
      const bool row_ok = r < m_used && t < rows_tok;
      const int tok = rec.t0 + x * tq + t;  // query token within the request
      const int64_t orow = static_cast<int64_t>(rec.q_start + tok) * p.hq + rec.h * g + jh;
      if (rec.n_tiles == 0) {  // no visible key: zeros, lse = -inf
        if (row_ok) {
          T *o = static_cast<T *>(p.out) + orow * D;
          for (int i = 0; i < D; ++i) o[i] = Elt<T>::from(0.f);
          if (p.lse) p.lse[orow] = -INFINITY;
        }
        continue;
      }
      int lim = p.causal ? rec.lk - rec.lq + tok + 1 : rec.lk;
      lim = min(lim, rec.lk);
      if (!row_ok) lim = 0;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < rec.n_tiles; ++j, ++gt) {
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[x], gt & 1))) { ok = false; break; }
        tc_fence_after();
        if (rows_tok == 0) {
          // a tile past its request's end: no products were issued for it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&p_full[x]);
          continue;
        }
        const int kbase = j * kN;
        // columns of S this tile computed: kN / 2 for a half tile (the
        // item's last, with at most kN / 2 visible keys)
        const int ncol = (j + 1 == rec.n_tiles && rec.last_keys <= kN / 2) ? kN / 2 : kN;
        const bool masked = __any_sync(0xffffffffu, kbase + ncol > lim);
        // S chunk c (32 keys) into registers, keys at or past lim as -inf
        auto load_chunk = [&](int c, float *sv) {
          tmem_ld32(tmem_s + c * 32, sv);
          tmem_wait_ld();
          if (masked) {
#pragma unroll
            for (int i = 0; i < 32; ++i) sv[i] = (kbase + c * 32 + i < lim) ? sv[i] : -INFINITY;
          }
        };
        float corr = 1.f, sum = 0.f, m_new = m;
        // the max the one pass works against: the running max, or in an
        // item's first tile the row max of its first 32 keys (key 0 is
        // visible to every row that sees any key)
        float mb = m;
        {
          // one pass against mb: P = 2^(s * scale - mb) chunk by chunk, each
          // chunk's P written over S columns already read. A chunk with a
          // key above mb + kRescaleLog2 (in a row of the warp) is not
          // written: from it on the tile takes two passes against a new
          // max, its S and the later chunks' being still in TMEM, and the P
          // already written (at most 2^kRescaleLog2, so it fits the 16-bit
          // type) is rebased. Row maxima and sums run in four independent
          // chains each, off the exponentials' path.
          float ms = mb == -INFINITY ? 0.f : mb;  // a row with no key yet
          float sm[4] = {0.f, 0.f, 0.f, 0.f};
          float cmax = -INFINITY;  // raw row max of the chunk the loop stopped at
          int c = 0;
#pragma unroll 1
          for (; c < ncol / 32; ++c) {
            float sv[32];
            load_chunk(c, sv);
            if (j == 0 && c == 0) {  // an item's first tile: mb from its first chunk
              float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
              for (int i = 0; i < 32; i += 4) {
                mx0 = max3f(mx0, sv[i], sv[i + 1]);
                mx1 = max3f(mx1, sv[i + 2], sv[i + 3]);
              }
              mb = fmaxf(mx0, mx1) * p.scale_log2;
              ms = mb == -INFINITY ? 0.f : mb;
            }
            float cm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            float cs[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              cm[(i >> 1) & 3] = max3f(cm[(i >> 1) & 3], sv[i], sv[i + 1]);
              const float p0 = fast_exp2(fmaf(sv[i], p.scale_log2, -ms));  // 2^-inf = 0
              const float p1 = fast_exp2(fmaf(sv[i + 1], p.scale_log2, -ms));
              cs[(i >> 1) & 3] += p0 + p1;
              pk[i >> 1] = Pack2<T>::run(p0, p1);
            }
            cmax = max3f(cm[0], cm[1], fmaxf(cm[2], cm[3]));
            if (__any_sync(0xffffffffu, cmax * p.scale_log2 > mb + kRescaleLog2)) break;
            tmem_st16(tmem_s + c * 16, pk);  // columns [16 c, 16 c + 16): read already
#pragma unroll
            for (int k = 0; k < 4; ++k) sm[k] += cs[k];
          }
          sum = (sm[0] + sm[1]) + (sm[2] + sm[3]);
          m_new = mb;  // (m itself after the first tile; O holds nothing before it)
          if (c < ncol / 32) {
            // pass 1 over chunk c and the rest: their row max (raw scores;
            // scale_log2 > 0, so the max commutes with it)
            float mt = cmax;
#pragma unroll 1
            for (int c2 = c + 1; c2 < ncol / 32; ++c2) {
              float sv[32];
              load_chunk(c2, sv);
#pragma unroll
              for (int i = 0; i < 32; ++i) mt = fmaxf(mt, sv[i]);
            }
            mt *= p.scale_log2;
            // keep mb unless they exceed it by more than kRescaleLog2
            m_new = (mt > mb + kRescaleLog2 || mb == -INFINITY) ? fmaxf(mb, mt) : mb;
            const float ms2 = m_new == -INFINITY ? 0.f : m_new;
            corr = m_new == mb ? 1.f : fast_exp2(mb - ms2);
            sum *= corr;
            // the P written for the chunks before c, rebased on m_new
            if (c > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll 1
              for (int c2 = 0; c2 < c; ++c2) {
                float pw[16];
                tmem_ld16(tmem_s + c2 * 16, pw);
                tmem_wait_ld();
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const float2 f = Unpack2<T>::run(__float_as_uint(pw[i]));
                  pk[i] = Pack2<T>::run(f.x * corr, f.y * corr);
                }
                tmem_st16(tmem_s + c2 * 16, pk);
              }
            }
            // pass 2: P of chunk c and the rest against m_new
#pragma unroll 1
            for (int c2 = c; c2 < ncol / 32; ++c2) {
              float sv[32];
              load_chunk(c2, sv);
              uint32_t pk[16];
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const float p0 = fast_exp2(fmaf(sv[i], p.scale_log2, -ms2));
                const float p1 = fast_exp2(fmaf(sv[i + 1], p.scale_log2, -ms2));
                sum += p0 + p1;
                pk[i >> 1] = Pack2<T>::run(p0, p1);
              }
              tmem_st16(tmem_s + c2 * 16, pk);
            }
          }
        }
        l = l * corr + sum;
        m = m_new;
        // rescale O (its previous P V is done: this tile's S was committed
        // after it)
        if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            float ov[16];
            tmem_ld16(tmem_o + c * 16, ov);
            tmem_wait_ld();
            uint32_t ou[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) ou[i] = __float_as_uint(ov[i] * corr);
            tmem_st16(tmem_o + c * 16, ou);
          }
        }
        tmem_wait_st();  // P (and a rescaled O) are in TMEM before the MMA is told
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
      }
      if (!ok) break;
      const int rows_a = max(0, min(tq, rec.lq - rec.t0));
      const int rows_b = max(0, min(tq, rec.lq - rec.t0 - tq));
      if (!hand_off(make_int4(rec.q_start + rec.t0, rec.h, rows_a, rows_b), l, m)) {
        ok = false;
        break;
      }
      ++oc;
    }
  } else {
    // ======================= epilogue (warps 10..13) =========================
    // Thread = TMEM lane = packed query row, all head_dim columns. Per item
    // and tile: wait for the tile's row sums (l_ready) and its last P V
    // (o_full), normalise O, store it, release the O buffer (o_free) and the
    // hand-off slot (h_free).
    const int qd = warp & 3;
    const int r = qd * 32 + lane;
    const int t = r / g, jh = r % g;
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const float *lsum = reinterpret_cast<const float *>(smem + L::LSUM_OFF);
    const float *mfin = reinterpret_cast<const float *>(smem + L::MFIN_OFF);
    const int4 *erec = reinterpret_cast<const int4 *>(smem + L::EREC_OFF);
    for (int oc = 0; ok; ++oc) {
      const int slot = oc & 1;
      int4 er = make_int4(0, 0, 0, 0);
      for (int x = 0; x < 2 && ok; ++x) {
        if (!__all_sync(0xffffffffu,
                        mbar_wait_bounded(&l_ready[slot * 2 + x], (oc >> 1) & 1))) {
          ok = false;
          break;
        }
        if (x == 0) {
          er = erec[slot];  // token base, KV head, query tokens of A and B; x < 0: the end
          if (er.x < 0) break;
        }
        const float l = lsum[(slot * 2 + x) * kM + r];
        const float m = mfin[(slot * 2 + x) * kM + r];
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&o_full[x], oc & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool row_ok = r < m_used && t < (x ? er.w : er.z);
        const int64_t orow = static_cast<int64_t>(er.x + x * tq + t) * p.hq + er.y * g + jh;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T *o = static_cast<T *>(p.out) + orow * D;
        const uint32_t tmem_o = tmem + L::O_COL + x * D + lane_base;
        auto store_chunk = [&](int c, const float *ov) {
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
        };
        // O in pairs of 32-column chunks, one TMEM round trip per pair; the
        // O buffer goes back to the MMA as soon as its last pair is read
#pragma unroll
        for (int c = 0; c < D / 32; c += 2) {
          float oa[32], ob[32];
          tmem_ld32(tmem_o + c * 32, oa);
          tmem_ld32(tmem_o + (c + 1) * 32, ob);
          tmem_wait_ld();
          if (c + 2 == D / 32) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[x]);  // O_x may be overwritten
          }
          store_chunk(c, oa);
          store_chunk(c + 1, ob);
        }
        if (row_ok && p.lse) p.lse[orow] = l > 0.f ? (m + __log2f(l)) * kLn2 : -INFINITY;
        __syncwarp();
        if (lane == 0) mbar_arrive(&h_free[slot * 2 + x]);  // the hand-off slot may be rewritten
      }
      if (!ok || er.x < 0) break;
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
int launch_t2(const PrefillParams &p, int dtype, cudaStream_t s) {
  using L = Pf2Layout<D>;
  CUtensorMap qmap, kvmap;
  const int tq = kM / p.group;
  if (!rows_tensor_map(p.q, p.total_q, p.hq, D, p.qsn, p.qsh, p.group, tq, dtype, &qmap))
    return -1;
  if (!pool_tensor_map(p.kv, p.num_pages, p.ps, p.hkv, D, dtype, &kvmap)) return -1;
  static std::atomic<unsigned long long> attr_set{0};
  if (smem_limit_once(attr_set, prefill_tc2_kernel<T, D>, L::SMEM) != cudaSuccess)
    return check_launch("prefill_tc2_kernel smem attribute");
  // persistent: one CTA per SM, or fewer when there are fewer work items
  // (an upper bound: (sum ceil(L_b / 2Tq)) * hkv <= (total / 2Tq + batch) * hkv)
  const int64_t items = (static_cast<int64_t>(p.total_q) / (2 * tq) + p.batch) * p.hkv;
  const int grid = static_cast<int>(std::min<int64_t>(items, num_sms()));
  prefill_tc2_kernel<T, D><<<grid, kThreads2, L::SMEM, s>>>(qmap, kvmap, p);
  return check_launch("prefill_tc2_kernel");
}

}  // namespace

int launch_prefill_tc2(const PrefillParams &p, int dtype, cudaStream_t s) {
  if (!(dtype == MI_DTYPE_BF16 || dtype == MI_DTYPE_F16)) return -1;
  if (!(p.d == 64 || p.d == 128)) return -1;
  if (p.group > kM || p.ps % 16 != 0 || p.ps > 256 || p.batch > kMaxBatch2) return -1;
  if (p.hkv > 65535 || p.num_pages * 2 > (1LL << 31)) return -1;
  if (!(p.scale_log2 > 0.f)) return -1;  // the softmax takes the row max before scaling
  if (static_cast<int64_t>(p.total_q) + 2 * kM > (1LL << 31)) return -1;
  if (dtype == MI_DTYPE_BF16)
    return p.d == 128 ? launch_t2<__nv_bfloat16, 128>(p, dtype, s)
                      : launch_t2<__nv_bfloat16, 64>(p, dtype, s);
  return p.d == 128 ? launch_t2<__half, 128>(p, dtype, s) : launch_t2<__half, 64>(p, dtype, s);
}

}  // namespace mi
