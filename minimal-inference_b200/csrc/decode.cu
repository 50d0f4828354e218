// Kernel (2): paged decode attention with native GQA and split-K.
//
// Replaces FlashInfer's BatchDecodeWithPagedKVCacheWrapper as the reference
// uses it (scheduler.py:535-539 ctor, :905-916 plan, model.py:235 run), and
// the GQA head padding/stripping around it (model.py:227-243).
//
// Fast path (bf16/fp16, head_dim 64/128, group <= 16): a persistent kernel
// whose warps are independent producer/consumer pipelines.
//   * Work unit ("item") = (request b, KV head h, chunk c of C tiles), a tile
//     being 16 consecutive tokens. Every CTA derives the same plan from
//     kv_indptr / kv_last_page_len in its prologue (no host plan(), so the
//     launch is CUDA-graph capturable); C is sized so the items cover the
//     grid's warps about twice. Warps take items from a global ticket.
//   * Streaming: each lane of a warp issues one bulk copy (TMA engine,
//     cp.async.bulk) of one 16-token row of K (lanes 0-15) or V (16-31)
//     straight from its page into a padded shared-memory tile; the tile's
//     mbarrier counts the bytes. Rows sit 16 bytes apart from a power-of-two
//     stride, so ldmatrix reads are bank-conflict free. S tiles per warp are
//     in flight.
//   * Math: mma.sync m16n8k16 with the group's query heads as the M rows
//     (no padding of the model; rows past the group are zero), S = Q K^T
//     and O += P V with P kept in registers; online softmax in the exp2
//     domain, row max / sum through quad shuffles.
//   * Split-K: an item that is not its request's only chunk writes a partial
//     (O normalised, log2-sum-exp) to the workspace; the last of the (b, h)
//     items to arrive (atomic counter) merges them and resets the counter.
// Generic path (any dtype incl. fp32, any head_dim <= 256): one CTA per
// (request, query head), warps split the tokens, online softmax per warp,
// merged through shared memory. Used for fp32 parity configs and shapes the
// fast path does not cover.
#include <cuda.h>

#include <mutex>

#include "decode_sk.cuh"
#include "mi_common.cuh"

namespace mi {
namespace {

struct DecodeParams {
  const void *q;
  int64_t qsb, qsh;
  const void *kv;
  int64_t num_pages;
  int ps, hkv, d;
  const int32_t *indptr, *indices, *last;
  int batch, hq, group;
  float scale_log2;  // sm_scale * log2(e)
  void *out;
  float *lse;
  int32_t *status;
  // workspace views (fast path)
  unsigned int *ctrl;    // [0] ticket, [1] warps done
  unsigned int *arrive;  // [batch * hkv] split-K arrival counters
  float *part_o;         // [max_items][group][d]
  float *part_lse;       // [max_items][group]
  int target_items, min_chunk_tiles;
};

constexpr int kTile = 16;     // tokens per tile
constexpr int kMaxBatch = 2048;  // fast path plan lives in shared memory

template <int D> struct TcCfg;
template <> struct TcCfg<128> {
  static constexpr int NW = 8, S = 3;
};
template <> struct TcCfg<64> {
  static constexpr int NW = 8, S = 5;
};

template <int D> struct TcLayout {
  static constexpr int NW = TcCfg<D>::NW, S = TcCfg<D>::S;
  static constexpr int ROW_BYTES = D * 2;
  static constexpr int ROW_STRIDE = ROW_BYTES + 16;
  static constexpr int STAGE_BYTES = 2 * kTile * ROW_STRIDE;  // K tile + V tile
  static constexpr int STAGES_BYTES = NW * S * STAGE_BYTES;
  static constexpr int BAR_OFF = STAGES_BYTES;
  static constexpr int REC_OFF = BAR_OFF + NW * S * 8;
  static constexpr int PLAN_OFF = REC_OFF + NW * S * 16;
  static constexpr int SMEM = PLAN_OFF + kMaxBatch * 4 + 16;
};

// Block-wide inclusive scan of per-request item counts into plan[].
// Returns the total. blockDim.x must be a multiple of 32.
__device__ int plan_items(const DecodeParams &p, int *plan, int *s_tmp, int chunk) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int carry = 0;
  for (int base = 0; base < p.batch; base += blockDim.x) {
    const int b = base + threadIdx.x;
    int n = 0;
    if (b < p.batch) {
      const int tiles = cdiv(kv_len_of(p.indptr, p.last, b, p.ps), kTile);
      n = cdiv(tiles, chunk) * p.hkv;
    }
    int x = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_tmp[warp] = x;
    __syncthreads();
    int wpre = 0, tot = 0;
    for (int w = 0; w < nw; ++w) {
      const int v = s_tmp[w];
      if (w < warp) wpre += v;
      tot += v;
    }
    if (b < p.batch) plan[b] = carry + wpre + x;
    carry += tot;
    __syncthreads();
  }
  return carry;
}

struct Item {
  int b, h, nch, tile0, tile_end, kvlen, page_base;
};

__device__ __forceinline__ Item decode_item(const DecodeParams &p, const int *plan, int it,
                                            int chunk) {
  int lo = 0, hi = p.batch - 1;
  while (lo < hi) {  // first b with plan[b] > it
    const int mid = (lo + hi) >> 1;
    if (plan[mid] > it) hi = mid; else lo = mid + 1;
  }
  Item r;
  r.b = lo;
  const int start = lo ? plan[lo - 1] : 0;
  r.nch = (plan[lo] - start) / p.hkv;
  const int local = it - start;
  r.h = local / r.nch;
  const int c = local - r.h * r.nch;
  r.kvlen = kv_len_of(p.indptr, p.last, lo, p.ps);
  const int tiles = cdiv(r.kvlen, kTile);
  r.tile0 = c * chunk;
  r.tile_end = min(tiles, r.tile0 + chunk);
  r.page_base = p.indptr[lo];
  return r;
}

template <typename T, int D, bool G16>
__global__ void __launch_bounds__(TcCfg<D>::NW * 32, 1) decode_tc_kernel(const DecodeParams p) {
  using L = TcLayout<D>;
  constexpr int NW = L::NW, S = L::S, KS = D / 16, NT = D / 8;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  int4 *recs = reinterpret_cast<int4 *>(smem + L::REC_OFF);
  int *plan = reinterpret_cast<int *>(smem + L::PLAN_OFF);
  __shared__ int s_tmp[32];
  __shared__ int s_total_tiles;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tq = lane & 3;
  const int total_warps = gridDim.x * NW;
  const int gwarp = blockIdx.x * NW + warp;

  // ---- prologue: barriers, zeroed tiles, plan ------------------------------
  if (threadIdx.x < NW * S) mbar_init(&bars[threadIdx.x], 1);
  {
    uint4 z = make_uint4(0, 0, 0, 0);
    uint4 *st = reinterpret_cast<uint4 *>(smem);
    for (int i = threadIdx.x; i < L::STAGES_BYTES / 16; i += blockDim.x) st[i] = z;
  }
  if (threadIdx.x == 0) s_total_tiles = 0;
  fence_mbar_init();
  __syncthreads();
  {
    int local = 0;
    for (int b = threadIdx.x; b < p.batch; b += blockDim.x)
      local += cdiv(kv_len_of(p.indptr, p.last, b, p.ps), kTile);
    local = __reduce_add_sync(0xffffffffu, local);
    if (lane == 0 && local) atomicAdd(&s_total_tiles, local);
  }
  __syncthreads();
  const int total_tiles = s_total_tiles;
  const int chunk = max(p.min_chunk_tiles,
                        cdiv(total_tiles * p.hkv, max(p.target_items, 1)));
  const int total_items = plan_items(p, plan, s_tmp, chunk);
  fence_proxy_async_smem();  // zeroed tiles visible to the async proxy
  __syncthreads();

  // requests with no tokens: zeros and lse = -inf (FlashInfer semantics)
  for (int b = gwarp; b < p.batch; b += total_warps) {
    if (kv_len_of(p.indptr, p.last, b, p.ps) != 0) continue;
    T *o = static_cast<T *>(p.out) + static_cast<int64_t>(b) * p.hq * D;
    for (int i = lane; i < p.hq * D; i += 32) o[i] = Elt<T>::from(0.f);
    if (p.lse)
      for (int i = lane; i < p.hq; i += 32) p.lse[b * p.hq + i] = -INFINITY;
  }

  unsigned char *my_stages = smem + warp * S * L::STAGE_BYTES;
  uint64_t *my_bars = bars + warp * S;
  int4 *my_recs = recs + warp * S;

  // ---- producer state ------------------------------------------------------
  unsigned int raw_ticket = 0;
  if (lane == 0) raw_ticket = atomicAdd(&p.ctrl[0], 1u);
  int p_item = -1, p_tile = 0;
  Item pi{};

  // Advance the producer to its next tile; false when the work is exhausted.
  auto p_advance = [&]() -> bool {
    if (p_item >= 0 && p_tile + 1 < pi.tile_end) {
      ++p_tile;
      return true;
    }
    const int t = __shfl_sync(0xffffffffu, static_cast<int>(raw_ticket), 0);
    if (t >= total_items) {
      p_item = total_items;  // exhausted; no further grabs
      return false;
    }
    if (lane == 0) raw_ticket = atomicAdd(&p.ctrl[0], 1u);  // prefetch the next ticket
    p_item = t;
    pi = decode_item(p, plan, t, chunk);
    p_tile = pi.tile0;
    return true;
  };

  const T *kvbase = static_cast<const T *>(p.kv);
  const int64_t slot_elems = static_cast<int64_t>(p.hkv) * D;
  // Issue the current producer tile into stage s.
  auto p_issue = [&](int s) {
    const int r = lane & 15, which = lane >> 4;
    const int t = p_tile * kTile + r;
    bool valid = t < pi.kvlen, bad = false;
    int64_t page = 0;
    int slot = 0;
    if (valid) {
      page = p.indices[pi.page_base + t / p.ps];
      slot = t % p.ps;
      if (page < 0 || page >= p.num_pages) valid = false, bad = true;
    }
    const unsigned int ball = __ballot_sync(0xffffffffu, valid);
    if (__any_sync(0xffffffffu, bad) && lane == 0) flag(p.status, MI_STATUS_BAD_PAGE);
    if (lane == 0) {
      my_recs[s] = make_int4(p_item, p_tile, static_cast<int>(ball & 0xffffu), 0);
      mbar_arrive_expect_tx(&my_bars[s], __popc(ball) * L::ROW_BYTES);
    }
    __syncwarp();
    if (valid) {
      const T *src = kvbase + ((page * 2 + which) * p.ps + slot) * slot_elems +
                     static_cast<int64_t>(pi.h) * D;
      unsigned char *dst = my_stages + s * L::STAGE_BYTES + (which * kTile + r) * L::ROW_STRIDE;
      bulk_g2s(dst, src, L::ROW_BYTES, &my_bars[s]);
    }
  };

  // ---- consumer state ------------------------------------------------------
  int c_item = -1;
  Item ci{};
  uint32_t qa[KS][4];
  float o[NT][4];
  float m0 = -INFINITY, l0 = 0.f, m1 = -INFINITY, l1 = 0.f;

  const uint32_t lane_k_off =
      (((lane >> 4) & 1) * 8 + (lane & 7)) * L::ROW_STRIDE + ((lane >> 3) & 1) * 16;
  const uint32_t lane_v_off =
      (((lane >> 3) & 1) * 8 + (lane & 7)) * L::ROW_STRIDE + ((lane >> 4) & 1) * 16;

  bool timed_out = false;
  int issued = 0, consumed = 0;
  for (int s = 0; s < S; ++s) {
    if (!p_advance()) break;
    p_issue(s);
    ++issued;
  }

  while (consumed < issued) {
    const int s = consumed % S;
    const uint32_t phase = (consumed / S) & 1;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&my_bars[s], phase))) {
      timed_out = true;
      break;
    }
    const int4 rec = my_recs[s];
    if (rec.x != c_item) {  // first tile of a new item: load its queries
      c_item = rec.x;
      ci = decode_item(p, plan, c_item, chunk);
      const T *qb = static_cast<const T *>(p.q) + static_cast<int64_t>(ci.b) * p.qsb;
      const int r0 = ci.h * p.group + gid;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const int dc = kk * 16 + 2 * tq;
        uint32_t a0 = 0, a2 = 0, a1 = 0, a3 = 0;
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
#pragma unroll
      for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
    }
    const uint32_t kbase = smem_u32(my_stages + s * L::STAGE_BYTES);
    const uint32_t vbase = kbase + kTile * L::ROW_STRIDE;

    // S = Q K^T over the 16 tokens of the tile
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(b0, b1, b2, b3, kbase + lane_k_off + kk * 32);
      Mma<T>::run(s0, qa[kk], b0, b1);
      Mma<T>::run(s1, qa[kk], b2, b3);
    }
    // online softmax (log2 domain); tokens 2t, 2t+1 | 8+2t, 9+2t of this lane
    const int nvalid = ci.kvlen - rec.y * kTile;
    const unsigned int vmask = static_cast<unsigned int>(rec.z);
    auto ok = [&](int tok) { return tok < nvalid && ((vmask >> tok) & 1u); };
    const int ta = 2 * tq, tb = 2 * tq + 1, tc = 8 + 2 * tq, td = 9 + 2 * tq;
    float x0 = ok(ta) ? s0[0] * p.scale_log2 : -INFINITY;
    float x1 = ok(tb) ? s0[1] * p.scale_log2 : -INFINITY;
    float x2 = ok(tc) ? s1[0] * p.scale_log2 : -INFINITY;
    float x3 = ok(td) ? s1[1] * p.scale_log2 : -INFINITY;
    float mx = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn0 = fmaxf(m0, mx);
    const float msafe0 = mn0 == -INFINITY ? 0.f : mn0;
    const float corr0 = exp2f(m0 - msafe0);
    const float p0 = exp2f(x0 - msafe0), p1 = exp2f(x1 - msafe0);
    const float p2 = exp2f(x2 - msafe0), p3 = exp2f(x3 - msafe0);
    l0 = l0 * corr0 + (p0 + p1 + p2 + p3);
    m0 = mn0;
    uint32_t pa[4];
    pa[0] = Mma<T>::pack(p0, p1);
    pa[2] = Mma<T>::pack(p2, p3);
    pa[1] = pa[3] = 0u;
    float corr1 = 1.f;
    if constexpr (G16) {
      float y0 = ok(ta) ? s0[2] * p.scale_log2 : -INFINITY;
      float y1 = ok(tb) ? s0[3] * p.scale_log2 : -INFINITY;
      float y2 = ok(tc) ? s1[2] * p.scale_log2 : -INFINITY;
      float y3 = ok(td) ? s1[3] * p.scale_log2 : -INFINITY;
      float my = fmaxf(fmaxf(y0, y1), fmaxf(y2, y3));
      my = fmaxf(my, __shfl_xor_sync(0xffffffffu, my, 1));
      my = fmaxf(my, __shfl_xor_sync(0xffffffffu, my, 2));
      const float mn1 = fmaxf(m1, my);
      const float msafe1 = mn1 == -INFINITY ? 0.f : mn1;
      corr1 = exp2f(m1 - msafe1);
      const float q0 = exp2f(y0 - msafe1), q1 = exp2f(y1 - msafe1);
      const float q2 = exp2f(y2 - msafe1), q3 = exp2f(y3 - msafe1);
      l1 = l1 * corr1 + (q0 + q1 + q2 + q3);
      m1 = mn1;
      pa[1] = Mma<T>::pack(q0, q1);
      pa[3] = Mma<T>::pack(q2, q3);
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      o[n][0] *= corr0;
      o[n][1] *= corr0;
      if constexpr (G16) {
        o[n][2] *= corr1;
        o[n][3] *= corr1;
      }
    }
    // O += P V
#pragma unroll
    for (int np = 0; np < KS; ++np) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(b0, b1, b2, b3, vbase + lane_v_off + np * 32);
      Mma<T>::run(o[2 * np], pa, b0, b1);
      Mma<T>::run(o[2 * np + 1], pa, b2, b3);
    }
    __syncwarp();
    fence_proxy_async_smem();
    ++consumed;
    if (p_advance()) {
      p_issue(s);
      ++issued;
    }

    if (rec.y + 1 == ci.tile_end) {  // last tile of the item: finalise
      float ls0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
      ls0 += __shfl_xor_sync(0xffffffffu, ls0, 2);
      float ls1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
      ls1 += __shfl_xor_sync(0xffffffffu, ls1, 2);
      const float inv0 = ls0 > 0.f ? 1.f / ls0 : 0.f;
      const float inv1 = ls1 > 0.f ? 1.f / ls1 : 0.f;
      const float lg0 = ls0 > 0.f ? m0 + __log2f(ls0) : -INFINITY;
      const float lg1 = ls1 > 0.f ? m1 + __log2f(ls1) : -INFINITY;
      const int row0 = gid, row1 = gid + 8;
      if (ci.nch == 1) {
        T *ob = static_cast<T *>(p.out) +
                (static_cast<int64_t>(ci.b) * p.hq + ci.h * p.group) * D;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          if (row0 < p.group)
            *reinterpret_cast<uint32_t *>(ob + row0 * D + n * 8 + 2 * tq) =
                Mma<T>::pack(o[n][0] * inv0, o[n][1] * inv0);
          if (G16 && row1 < p.group)
            *reinterpret_cast<uint32_t *>(ob + row1 * D + n * 8 + 2 * tq) =
                Mma<T>::pack(o[n][2] * inv1, o[n][3] * inv1);
        }
        if (p.lse && tq == 0) {
          const int base = ci.b * p.hq + ci.h * p.group;
          if (row0 < p.group) p.lse[base + row0] = lg0 * kLn2;
          if (G16 && row1 < p.group) p.lse[base + row1] = lg1 * kLn2;
        }
      } else {
        float *po = p.part_o + static_cast<int64_t>(c_item) * p.group * D;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          if (row0 < p.group)
            *reinterpret_cast<float2 *>(po + row0 * D + n * 8 + 2 * tq) =
                make_float2(o[n][0] * inv0, o[n][1] * inv0);
          if (G16 && row1 < p.group)
            *reinterpret_cast<float2 *>(po + row1 * D + n * 8 + 2 * tq) =
                make_float2(o[n][2] * inv1, o[n][3] * inv1);
        }
        if (tq == 0) {
          if (row0 < p.group) p.part_lse[c_item * p.group + row0] = lg0;
          if (G16 && row1 < p.group) p.part_lse[c_item * p.group + row1] = lg1;
        }
        __threadfence();
        __syncwarp();
        unsigned int prev = 0;
        unsigned int *cnt = &p.arrive[ci.b * p.hkv + ci.h];
        if (lane == 0) prev = atomicAdd(cnt, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev + 1 == static_cast<unsigned int>(ci.nch)) {
          // last arrival: merge every chunk of (b, h)
          __threadfence();
          const int start = c_item - (c_item - (ci.b ? plan[ci.b - 1] : 0)) % ci.nch;
          constexpr int DPL = D / 32;
          T *ob = static_cast<T *>(p.out) +
                  (static_cast<int64_t>(ci.b) * p.hq + ci.h * p.group) * D;
          for (int r = 0; r < p.group; ++r) {
            float M = -INFINITY;
            for (int c = 0; c < ci.nch; ++c)
              M = fmaxf(M, __ldcg(p.part_lse + (start + c) * p.group + r));
            float acc[DPL];
#pragma unroll
            for (int j = 0; j < DPL; ++j) acc[j] = 0.f;
            float wsum = 0.f;
            if (M != -INFINITY) {
              for (int c = 0; c < ci.nch; ++c) {
                const float w = exp2f(__ldcg(p.part_lse + (start + c) * p.group + r) - M);
                wsum += w;
                const float *src = p.part_o + (static_cast<int64_t>(start + c) * p.group + r) * D;
#pragma unroll
                for (int j = 0; j < DPL; ++j) acc[j] += w * __ldcg(src + j * 32 + lane);
              }
            }
            const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
#pragma unroll
            for (int j = 0; j < DPL; ++j) ob[r * D + j * 32 + lane] = Elt<T>::from(acc[j] * inv);
            if (p.lse && lane == 0)
              p.lse[ci.b * p.hq + ci.h * p.group + r] =
                  wsum > 0.f ? (M + __log2f(wsum)) * kLn2 : -INFINITY;
          }
          if (lane == 0) *cnt = 0u;
        }
      }
    }
  }

  if (timed_out) {
    flag(p.status, MI_STATUS_TIMEOUT);
    // let the copies still in flight land before the CTA's shared memory goes
    for (int k = consumed + 1; k < issued; ++k)
      (void)mbar_wait_bounded(&my_bars[k % S], (k / S) & 1);
  }
  // last warp out resets the ticket for the next launch
  if (lane == 0) {
    __threadfence();
    if (atomicAdd(&p.ctrl[1], 1u) + 1 == static_cast<unsigned int>(total_warps)) {
      p.ctrl[0] = 0u;
      p.ctrl[1] = 0u;
    }
  }
}

// ---------------------------------------------------------------------------
// generic path: one CTA per (request, query head)
// ---------------------------------------------------------------------------
template <typename T, int DPL>
__global__ void __launch_bounds__(128) decode_generic_kernel(const DecodeParams p) {
  constexpr int NWG = 4;
  const int b = blockIdx.x, hqi = blockIdx.y, h = hqi / p.group;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ float s_m[NWG], s_l[NWG];
  __shared__ float s_acc[NWG][DPL * 32];
  const int kvlen = kv_len_of(p.indptr, p.last, b, p.ps);
  const T *qr = static_cast<const T *>(p.q) + static_cast<int64_t>(b) * p.qsb +
                static_cast<int64_t>(hqi) * p.qsh;
  float qv[DPL], acc[DPL];
#pragma unroll
  for (int j = 0; j < DPL; ++j) {
    const int dd = j * 32 + lane;
    qv[j] = dd < p.d ? Elt<T>::to(qr[dd]) : 0.f;
    acc[j] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const T *kv = static_cast<const T *>(p.kv);
  const int64_t slot_elems = static_cast<int64_t>(p.hkv) * p.d;
  for (int t = warp; t < kvlen; t += NWG) {
    const int64_t page = p.indices[p.indptr[b] + t / p.ps];
    if (page < 0 || page >= p.num_pages) {
      if (lane == 0) flag(p.status, MI_STATUS_BAD_PAGE);
      continue;
    }
    const T *kr = kv + ((page * 2) * p.ps + t % p.ps) * slot_elems + static_cast<int64_t>(h) * p.d;
    const T *vr = kr + static_cast<int64_t>(p.ps) * slot_elems;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int dd = j * 32 + lane;
      if (dd < p.d) s += qv[j] * Elt<T>::to(kr[dd]);
    }
    s = warp_sum(s) * p.scale_log2;
    const float mn = fmaxf(m, s);
    const float corr = exp2f(m - mn);
    const float pr = exp2f(s - mn);
    l = l * corr + pr;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int dd = j * 32 + lane;
      acc[j] = acc[j] * corr + (dd < p.d ? pr * Elt<T>::to(vr[dd]) : 0.f);
    }
    m = mn;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
#pragma unroll
  for (int j = 0; j < DPL; ++j) s_acc[warp][j * 32 + lane] = acc[j];
  __syncthreads();
  if (warp == 0) {
    float M = -INFINITY;
    for (int w = 0; w < NWG; ++w) M = fmaxf(M, s_m[w]);
    float den = 0.f, num[DPL];
#pragma unroll
    for (int j = 0; j < DPL; ++j) num[j] = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < NWG; ++w) {
        const float c = exp2f(s_m[w] - M);
        den += c * s_l[w];
#pragma unroll
        for (int j = 0; j < DPL; ++j) num[j] += c * s_acc[w][j * 32 + lane];
      }
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
    T *orow = static_cast<T *>(p.out) + (static_cast<int64_t>(b) * p.hq + hqi) * p.d;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int dd = j * 32 + lane;
      if (dd < p.d) orow[dd] = Elt<T>::from(num[j] * inv);
    }
    if (p.lse && lane == 0)
      p.lse[b * p.hq + hqi] = den > 0.f ? (M + __log2f(den)) * kLn2 : -INFINITY;
  }
}

template <typename T>
int launch_generic(const DecodeParams &p, cudaStream_t s) {
  dim3 grid(p.batch, p.hq);
  if (p.d <= 32) decode_generic_kernel<T, 1><<<grid, 128, 0, s>>>(p);
  else if (p.d <= 64) decode_generic_kernel<T, 2><<<grid, 128, 0, s>>>(p);
  else if (p.d <= 128) decode_generic_kernel<T, 4><<<grid, 128, 0, s>>>(p);
  else decode_generic_kernel<T, 8><<<grid, 128, 0, s>>>(p);
  return check_launch("decode_generic_kernel");
}

// Workspace layout of the fast path.
constexpr size_t kCtrlBytes = 256;
inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int fast_max_items(int batch, int hkv) {
  // two items per resident warp plus one partial chunk per (request, head)
  return 2 * num_sms() * 8 + batch * hkv;
}

size_t fast_ws_bytes(int batch, int hq, int hkv, int d, int max_items) {
  const int group = hq / hkv;
  return kCtrlBytes + align256(size_t(batch) * hkv * 4) +
         align256(size_t(max_items) * group * d * 4) + align256(size_t(max_items) * group * 4);
}

template <typename T, int D, bool G16>
int launch_tc(DecodeParams p, void *ws, size_t ws_bytes, cudaStream_t s) {
  using L = TcLayout<D>;
  static std::atomic<unsigned long long> attr_set{0};
  if (smem_limit_once(attr_set, decode_tc_kernel<T, D, G16>, L::SMEM) != cudaSuccess)
    return check_launch("decode_tc_kernel smem attribute");
  const int group = p.hq / p.hkv;
  unsigned char *w = static_cast<unsigned char *>(ws);
  p.ctrl = reinterpret_cast<unsigned int *>(w);
  p.arrive = reinterpret_cast<unsigned int *>(w + kCtrlBytes);
  const size_t arrive_bytes = align256(size_t(p.batch) * p.hkv * 4);
  // the rest of the workspace holds as many partial slots as fit
  const size_t per_item = size_t(group) * D * 4 + size_t(group) * 4;
  const size_t rest = ws_bytes > kCtrlBytes + arrive_bytes + 512 ? ws_bytes - kCtrlBytes - arrive_bytes - 512 : 0;
  const long long max_items = static_cast<long long>(rest / per_item);
  p.part_o = reinterpret_cast<float *>(w + kCtrlBytes + arrive_bytes);
  p.part_lse = reinterpret_cast<float *>(
      w + kCtrlBytes + arrive_bytes + align256(size_t(max_items) * group * D * 4));
  const int grid = num_sms();
  const long long room = max_items - static_cast<long long>(p.batch) * p.hkv;
  if (room < 1)
    return fail(MI_ERR_WORKSPACE, "decode: workspace of %zu bytes too small for batch %d",
                ws_bytes, p.batch);
  p.target_items = static_cast<int>(room < 2LL * grid * L::NW ? room : 2LL * grid * L::NW);
  p.min_chunk_tiles = 4;
  decode_tc_kernel<T, D, G16><<<grid, L::NW * 32, L::SMEM, s>>>(p);
  return check_launch("decode_tc_kernel");
}

// Shapes and alignments the workspace kernels (stream-K, then the ticket
// kernel) serve; every other call runs the generic kernel, which needs no
// workspace.
bool decode_fast_shape(const void *q, int64_t qsb, int64_t qsh, const void *kv, const void *out,
                       int head_dim, int dtype, int group, int batch) {
  const bool half_type = dtype == MI_DTYPE_BF16 || dtype == MI_DTYPE_F16;
  const bool aligned = (reinterpret_cast<uintptr_t>(q) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(kv) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(out) % 16 == 0) && qsb % 8 == 0 &&
                       qsh % 8 == 0;
  return half_type && (head_dim == 64 || head_dim == 128) && group <= 16 && batch <= kMaxBatch &&
         aligned;
}

template <typename T>
int launch_fast(const DecodeParams &p, void *ws, size_t ws_bytes, cudaStream_t s) {
  const bool g16 = p.group > 8;
  if (p.d == 128)
    return g16 ? launch_tc<T, 128, true>(p, ws, ws_bytes, s) : launch_tc<T, 128, false>(p, ws, ws_bytes, s);
  return g16 ? launch_tc<T, 64, true>(p, ws, ws_bytes, s) : launch_tc<T, 64, false>(p, ws, ws_bytes, s);
}

}  // namespace
}  // namespace mi

extern "C" size_t mi_paged_decode_workspace_size(int32_t batch_size, int32_t num_qo_heads,
                                                 int32_t num_kv_heads, int32_t head_dim) {
  using namespace mi;
  if (batch_size <= 0 || num_kv_heads <= 0 || num_qo_heads < num_kv_heads || head_dim <= 0)
    return 0;
  const size_t v1 = fast_ws_bytes(batch_size, num_qo_heads, num_kv_heads, head_dim,
                                 fast_max_items(batch_size, num_kv_heads)) + 512;
  const size_t sk = decode_sk_workspace_bytes(batch_size, num_qo_heads, num_kv_heads, head_dim);
  return v1 > sk ? v1 : sk;
}

extern "C" int mi_paged_decode(
    const void *q, int64_t q_stride_b, int64_t q_stride_h,
    const void *kv_data, int64_t num_pages, int32_t page_size, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype,
    const int32_t *kv_indptr, const int32_t *kv_indices, const int32_t *kv_last_page_len,
    int32_t batch_size, int32_t num_qo_heads, float sm_scale,
    void *out, float *lse, void *workspace, size_t workspace_bytes, int32_t *status,
    mi_stream_t stream) {
  using namespace mi;
  MI_REQUIRE(batch_size >= 0, "decode: negative batch_size");
  if (batch_size == 0) return MI_OK;
  MI_REQUIRE(q && kv_data && kv_indptr && kv_indices && kv_last_page_len && out,
             "decode: null pointer argument");
  MI_REQUIRE(page_size > 0 && num_kv_heads > 0 && head_dim > 0 && num_pages > 0,
             "decode: bad pool geometry");
  MI_REQUIRE(num_qo_heads >= num_kv_heads && num_qo_heads % num_kv_heads == 0,
             "decode: num_qo_heads %d is not a multiple of num_kv_heads %d", num_qo_heads,
             num_kv_heads);
  MI_REQUIRE(head_dim <= 256, "decode: head_dim %d > 256 unsupported", head_dim);
  MI_REQUIRE(dtype == MI_DTYPE_F32 || dtype == MI_DTYPE_F16 || dtype == MI_DTYPE_BF16,
             "decode: bad dtype %d", dtype);
  DecodeParams p{};
  p.q = q;
  p.qsb = q_stride_b;
  p.qsh = q_stride_h;
  p.kv = kv_data;
  p.num_pages = num_pages;
  p.ps = page_size;
  p.hkv = num_kv_heads;
  p.d = head_dim;
  p.indptr = kv_indptr;
  p.indices = kv_indices;
  p.last = kv_last_page_len;
  p.batch = batch_size;
  p.hq = num_qo_heads;
  p.group = num_qo_heads / num_kv_heads;
  p.scale_log2 = sm_scale * kLog2e;
  p.out = out;
  p.lse = lse;
  p.status = status;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool fast = workspace != nullptr &&
                    decode_fast_shape(q, q_stride_b, q_stride_h, kv_data, out, head_dim, dtype,
                                      num_qo_heads / num_kv_heads, batch_size);
  if (fast) {
    MI_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0,
               "decode: workspace must be 256-byte aligned");
    // stream-K TMA kernel first; the persistent ticket kernel covers the rest
    SkArgs sk{q, q_stride_b, q_stride_h, kv_data, num_pages, page_size, num_kv_heads,
              head_dim, dtype, kv_indptr, kv_indices, kv_last_page_len, batch_size,
              num_qo_heads, sm_scale, out, lse, workspace, workspace_bytes, status, s};
    const int rc = launch_decode_sk(sk);
    if (rc >= 0) return rc;
    return dtype == MI_DTYPE_BF16 ? launch_fast<__nv_bfloat16>(p, workspace, workspace_bytes, s)
                                  : launch_fast<__half>(p, workspace, workspace_bytes, s);
  }
  switch (dtype) {
    case MI_DTYPE_F32: return launch_generic<float>(p, s);
    case MI_DTYPE_F16: return launch_generic<__half>(p, s);
    default: return launch_generic<__nv_bfloat16>(p, s);
  }
}

// ---------------------------------------------------------------------------
// Decode step with the append fused in: request b's new token (position
// kv_len_b - 1) is rotated and written into its page by the decode kernel
// itself, and the raw queries are rotated as they are loaded. Same result as
// mi_append_paged_kv_cache(k_new, v_new, batch_indices = 0..B-1, positions =
// kv_len - 1, rope tables, q, q_out) followed by mi_paged_decode(q_out),
// bit for bit, in one launch pair instead of three launches. Only the
// stream-K kernel does it: other shapes return MI_ERR_UNSUPPORTED and launch
// nothing, and the caller makes the two calls.
// ---------------------------------------------------------------------------
extern "C" int mi_paged_decode_append(
    const void *q, int64_t q_stride_b, int64_t q_stride_h,
    const void *k_new, int64_t k_stride_b, int64_t k_stride_h,
    const void *v_new, int64_t v_stride_b, int64_t v_stride_h,
    const void *rope_cos, const void *rope_sin, int32_t rope_max_pos,
    void *kv_data, int64_t num_pages, int32_t page_size, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype,
    const int32_t *kv_indptr, const int32_t *kv_indices, const int32_t *kv_last_page_len,
    int32_t batch_size, int32_t num_qo_heads, float sm_scale,
    void *out, float *lse, void *workspace, size_t workspace_bytes, int32_t *status,
    mi_stream_t stream) {
  using namespace mi;
  MI_REQUIRE(batch_size >= 0, "decode_append: negative batch_size");
  if (batch_size == 0) return MI_OK;
  MI_REQUIRE(q && k_new && v_new && rope_cos && rope_sin && kv_data && kv_indptr &&
                 kv_indices && kv_last_page_len && out && workspace,
             "decode_append: null pointer argument");
  MI_REQUIRE(page_size > 0 && num_kv_heads > 0 && head_dim > 0 && num_pages > 0 &&
                 rope_max_pos > 0,
             "decode_append: bad pool geometry or RoPE table length");
  MI_REQUIRE(num_qo_heads >= num_kv_heads && num_qo_heads % num_kv_heads == 0,
             "decode_append: num_qo_heads %d is not a multiple of num_kv_heads %d",
             num_qo_heads, num_kv_heads);
  MI_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0,
             "decode_append: workspace must be 256-byte aligned");
  const bool half_type = dtype == MI_DTYPE_BF16 || dtype == MI_DTYPE_F16;
  if (!(half_type && (head_dim == 64 || head_dim == 128) &&
        num_qo_heads / num_kv_heads <= 16 && batch_size <= kMaxBatch &&
        reinterpret_cast<uintptr_t>(out) % 16 == 0))
    return fail(MI_ERR_UNSUPPORTED, "decode_append: shape outside the fused kernel's coverage");
  SkArgs sk{q, q_stride_b, q_stride_h, kv_data, num_pages, page_size, num_kv_heads,
            head_dim, dtype, kv_indptr, kv_indices, kv_last_page_len, batch_size,
            num_qo_heads, sm_scale, out, lse, workspace, workspace_bytes, status,
            reinterpret_cast<cudaStream_t>(stream)};
  sk.k_new = k_new;
  sk.ksb = k_stride_b;
  sk.ksh = k_stride_h;
  sk.v_new = v_new;
  sk.vsb = v_stride_b;
  sk.vsh = v_stride_h;
  sk.rope_cos = rope_cos;
  sk.rope_sin = rope_sin;
  sk.rope_max = rope_max_pos;
  const int rc = launch_decode_sk(sk);
  if (rc >= 0) return rc;
  return fail(MI_ERR_UNSUPPORTED,
              "decode_append: shape, alignment or workspace outside the fused kernel's coverage");
}

// ---------------------------------------------------------------------------
// Paged decode for callers that cannot allocate device memory.
//
// Some hosts own every byte of GPU memory through their own allocator (a
// serving runtime's caching pool, a fixed arena handed to plugins) and give a
// kernel library no way to obtain a workspace; others call in from places
// where a cudaMalloc is not allowed or would stall the whole device. For them
// the split-K scratch lives in a fixed array inside this library instead of a
// caller-provided workspace. Every GPU that loads the library holds the array
// until the process exits.
// ---------------------------------------------------------------------------
namespace mi {

static __device__ __align__(256) unsigned char g_decode_scratch[MI_DECODE_STATIC_SCRATCH_BYTES];

namespace {

constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mu;
struct ScratchSlot {
  CUcontext ctx;  // the context the address belongs to
  void *addr;
};
ScratchSlot g_scratch[kMaxScratchDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext *);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  return fn;
}

// Device address of g_decode_scratch on the current device. Looked up with
// that device current and cached together with its context, so a device
// reset (a new context, the array registered anew) makes the next call look
// it up again; in host code the array's name is only a stand-in, never a
// usable pointer.
int scratch_address(void **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(MI_ERR_CUDA, "decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxScratchDevices)
    return fail(MI_ERR_UNSUPPORTED, "decode_noalloc: device %d beyond %d", dev,
                kMaxScratchDevices);
  // the runtime makes the device's primary context current on first use
  e = cudaFree(nullptr);
  if (e != cudaSuccess)
    return fail(MI_ERR_CUDA, "decode_noalloc: context set-up: %s", cudaGetErrorString(e));
  CUcontext ctx = nullptr;
  auto get_ctx = ctx_get_current_fn();
  if (get_ctx == nullptr || get_ctx(&ctx) != CUDA_SUCCESS)
    return fail(MI_ERR_CUDA, "decode_noalloc: cuCtxGetCurrent unavailable");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot &slot = g_scratch[dev];
  if (slot.addr == nullptr || slot.ctx != ctx) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(MI_ERR_CUDA, "decode_noalloc: cudaGetSymbolAddress: %s",
                  cudaGetErrorString(e));
    slot.ctx = ctx;
    slot.addr = p;
  }
  *out = slot.addr;
  return MI_OK;
}

}  // namespace
}  // namespace mi

extern "C" int mi_paged_decode_noalloc(
    const void *q, int64_t q_stride_b, int64_t q_stride_h,
    const void *kv_data, int64_t num_pages, int32_t page_size, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype,
    const int32_t *kv_indptr, const int32_t *kv_indices, const int32_t *kv_last_page_len,
    int32_t batch_size, int32_t num_qo_heads, float sm_scale,
    void *out, float *lse, int32_t *status, mi_stream_t stream) {
  using namespace mi;
  MI_REQUIRE(batch_size >= 0, "decode_noalloc: negative batch_size");
  if (batch_size == 0) return MI_OK;
  MI_REQUIRE(num_kv_heads > 0 && head_dim > 0 && num_qo_heads >= num_kv_heads &&
                 num_qo_heads % num_kv_heads == 0,
             "decode_noalloc: bad head counts %d / %d", num_qo_heads, num_kv_heads);
  // Calls outside the workspace kernels' shapes run the generic kernel,
  // which uses no scratch: no limit applies to them.
  if (!decode_fast_shape(q, q_stride_b, q_stride_h, kv_data, out, head_dim, dtype,
                         num_qo_heads / num_kv_heads, batch_size))
    return mi_paged_decode(q, q_stride_b, q_stride_h, kv_data, num_pages, page_size,
                           num_kv_heads, head_dim, dtype, kv_indptr, kv_indices,
                           kv_last_page_len, batch_size, num_qo_heads, sm_scale, out, lse,
                           nullptr, 0, status, stream);
  // Room for the counters plus at least one partial slot per (request, KV
  // head); anything larger than the fixed array is refused here.
  const size_t group = static_cast<size_t>(num_qo_heads / num_kv_heads);
  const size_t counters = kCtrlBytes + align256(size_t(batch_size) * num_kv_heads * 4);
  const size_t per_item = group * head_dim * 4 + group * 4;
  const size_t need = counters + 512 + (size_t(batch_size) * num_kv_heads + 1) * per_item;
  if (need > MI_DECODE_STATIC_SCRATCH_BYTES)
    return fail(MI_ERR_WORKSPACE,
                "decode_noalloc: batch %d x %d KV heads needs %zu bytes of scratch, more than "
                "the library's fixed %u bytes; use mi_paged_decode with a workspace",
                batch_size, num_kv_heads, need, (unsigned)MI_DECODE_STATIC_SCRATCH_BYTES);
  void *scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != MI_OK) return rc;
  // The array keeps the previous call's contents: clear the counters the
  // kernel expects at zero (partial slots are written before they are read).
  cudaError_t e = cudaMemsetAsync(scratch, 0, counters, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(MI_ERR_CUDA, "decode_noalloc: clearing scratch: %s", cudaGetErrorString(e));
  return mi_paged_decode(q, q_stride_b, q_stride_h, kv_data, num_pages, page_size, num_kv_heads,
                         head_dim, dtype, kv_indptr, kv_indices, kv_last_page_len, batch_size,
                         num_qo_heads, sm_scale, out, lse, scratch,
                         MI_DECODE_STATIC_SCRATCH_BYTES, status, stream);
}
