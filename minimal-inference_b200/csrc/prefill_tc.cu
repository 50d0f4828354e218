// Kernel (3), tensor-core path: paged prefill attention on tcgen05 / TMEM.
//
// Replaces the FlashInfer fa2 prefill the reference runs (mma.sync,
// scheduler.py:530-534, :704-716, model.py:235) for bf16/fp16, head_dim
// 64/128, page_size a multiple of 16.
//
// CTA = (request, KV head, 128 "packed" query rows): a row is a (query token,
// query head of the GQA group) pair, row = token * group + head, so one K/V
// tile feeds the whole group (Tq = 128 / group tokens per CTA). Six warps:
//   warp 0  producer: TMA loads of the Q tile (3-D map over q) and of 128-token
//           K/V tiles straight from the pages (4-D pool map, 16-token boxes),
//           two K/V stages, 128-byte swizzle;
//   warp 1  MMA issuer (one thread): S = Q K^T into TMEM (M=128, N=128,
//           K=head_dim, both operands K-major), then O += P V into TMEM
//           (P K-major from shared memory, V MN-major), tcgen05.commit to
//           mbarriers. S of tile j+1 is issued as soon as the softmax warps
//           hold S of tile j in registers, so it runs under their softmax;
//           P V of tile j follows once P is written;
//   warps 2-5  softmax and epilogue: thread = TMEM lane = query row. Each KV
//           tile: load the S row, causal/length mask, online softmax in the
//           exp2 domain, write the bf16 P row into a 128-byte-swizzled tile,
//           rescale the O row in TMEM when the row max moved; at the end
//           normalise O and store it.
// TMEM: S in columns [0,128), O in [128, 128+head_dim). Every wait is
// bounded; TMEM is freed on every path.
#include <type_traits>

#include "prefill.cuh"
#include "tma.cuh"

namespace mi {
namespace {

constexpr int kM = 128;       // packed query rows per CTA
constexpr int kN = 128;       // KV tokens per tile
constexpr int kThreadsP = 192;
constexpr int kMaxBatchTc = 1024;

template <int D> struct PfLayout {
  static constexpr int DH = D / 64;                   // 64-wide blocks of head_dim
  static constexpr int Q_BYTES = DH * kM * 128;       // [dh][row][64]
  static constexpr int K_BYTES = DH * kN * 128;       // [dh][token][64]
  static constexpr int V_BYTES = K_BYTES;
  static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  static constexpr int P_BYTES = (kN / 64) * kM * 128;  // [kblock][row][64]
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = Q_OFF + Q_BYTES;
  static constexpr int P_OFF = KV_OFF + 2 * STAGE_BYTES;
  static constexpr int BAR_OFF = P_OFF + P_BYTES;      // 10 mbarriers + tmem base
  static constexpr int META_OFF = BAR_OFF + 128;
  static constexpr int SMEM = META_OFF + (kMaxBatchTc + 1) * 4 + 1024;
};

// UMMA shared-memory descriptor, 128-byte swizzle (sm100 layout): start >> 4
// [0,14), leading byte offset >> 4 [16,30), stride byte offset >> 4 [32,46),
// version 1 [46,48), layout type 2 = SWIZZLE_128B [61,64).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFF) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}

// kind::f16 instruction descriptor: f32 accumulate, A/B format (0 f16,
// 1 bf16), A K-major, B K- or MN-major, N, M.
__host__ __device__ constexpr uint32_t umma_idesc(uint32_t fmt, bool b_mn, int n, int m) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                     uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <typename T> struct Pack2;
template <> struct Pack2<__nv_bfloat16> {
  __device__ __forceinline__ static uint32_t run(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};
template <> struct Pack2<__half> {
  __device__ __forceinline__ static uint32_t run(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreadsP, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kvmap, const PrefillParams p) {
  using L = PfLayout<D>;
  constexpr int DH = L::DH;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  uint64_t *q_full = bars + 0, *kv_full = bars + 1, *kv_empty = bars + 3;
  uint64_t *s_full = bars + 5, *s_free = bars + 6, *p_full = bars + 7, *o_done = bars + 8;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 10);
  int *tiles_pre = reinterpret_cast<int *>(smem + L::META_OFF);
  __shared__ int s_info[2];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int g = p.group;
  const int tq = kM / g;        // query tokens per CTA
  const int m_used = tq * g;    // packed rows in use

  // ---- which request / query tile is this CTA ------------------------------
  if (warp == 0) {  // tiles_pre[i] = sum over b < i of ceil(qo_len_b / tq)
    int carry = 0;
    if (lane == 0) tiles_pre[0] = 0;
    for (int base = 0; base < p.batch; base += 32) {
      const int bb = base + lane;
      int x = bb < p.batch ? cdiv(p.qo_indptr[bb + 1] - p.qo_indptr[bb], tq) : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (bb < p.batch) tiles_pre[bb + 1] = carry + x;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int tile = blockIdx.x;
    int b = -1;
    if (tile < tiles_pre[p.batch]) {
      int lo = 0, hi = p.batch - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (tiles_pre[mid] <= tile) lo = mid; else hi = mid - 1;
      }
      b = lo;
    }
    s_info[0] = b;
    s_info[1] = b >= 0 ? (tile - tiles_pre[b]) * tq : 0;
  }
  __syncthreads();
  const int b = s_info[0];
  if (b < 0) return;  // past the last query tile
  const int t0 = s_info[1];
  const int q_start = p.qo_indptr[b];
  const int lq = p.qo_indptr[b + 1] - q_start;
  const int lk = kv_len_of(p.indptr, p.last, b, p.ps);
  const int rows_tok = min(tq, lq - t0);
  int lim_tok = p.causal ? min(lk, lk - lq + t0 + rows_tok) : lk;
  const int n_tiles = lim_tok > 0 ? cdiv(lim_tok, kN) : 0;

  if (n_tiles == 0) {  // no visible key: zeros, lse = -inf (warps 2..5)
    if (warp >= 2) {
      const int r = (warp & 3) * 32 + lane;
      const int t = r / g, j = r % g;
      if (r < m_used && t < rows_tok) {
        T *o = static_cast<T *>(p.out) +
               (static_cast<int64_t>(q_start + t0 + t) * p.hq + h * g + j) * D;
        for (int i = 0; i < D; ++i) o[i] = Elt<T>::from(0.f);
        if (p.lse) p.lse[static_cast<int64_t>(q_start + t0 + t) * p.hq + h * g + j] = -INFINITY;
      }
    }
    return;
  }

  // ---- setup: barriers, zeroed V stages, TMEM ------------------------------
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(&kv_full[0], 1);
    mbar_init(&kv_full[1], 1);
    mbar_init(&kv_empty[0], 1);
    mbar_init(&kv_empty[1], 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_mbar_init();
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_s = tmem, tmem_o = tmem + kN;
  bool ok = true;

  if (warp == 0) {
    // ============================ producer ==================================
    const uint64_t pol_q = evict_last_policy(), pol_kv = evict_first_policy();
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, DH * m_used * 128);
      for (int dh = 0; dh < DH; ++dh)
        tma_load_3d(smem + L::Q_OFF + dh * kM * 128, &qmap, dh * 64, h * g, q_start + t0, q_full,
                    pol_q);
    }
    const int page_base = p.indptr[b];
    const int nbox = 8 * 2 * DH;  // (16-token chunk, K/V, d block)
    for (int j = 0; j < n_tiles && ok; ++j) {
      const int s = j & 1;
      const int tok_tile = j * kN;
      // page id of chunk c = lane (c < 8)
      const int tok_c = tok_tile + lane * 16;
      int pg = -1;
      if (lane < 8 && tok_c < lk) pg = p.indices[page_base + tok_c / p.ps];
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&kv_empty[s], ((j >> 1) & 1) ^ 1))) {
        ok = false;
        break;
      }
      const int nvc = min(8, cdiv(lk - tok_tile, 16));
      if (j < 2 && nvc < 8) {
        // V chunks past the request's end are multiplied by P = 0; on a
        // stage's first use they hold whatever shared memory held, so zero
        // them (later uses keep the previous tile's finite values there)
        for (int dh = 0; dh < DH; ++dh) {
          uint4 *v = reinterpret_cast<uint4 *>(smem + L::KV_OFF + s * L::STAGE_BYTES +
                                               L::K_BYTES + dh * (kN * 128) + nvc * 16 * 128);
          for (int i = lane; i < (8 - nvc) * 16 * 128 / 16; i += 32) v[i] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();  // the zeros are visible to the tensor core
        __syncwarp();
      }
      if (lane == 0) mbar_arrive_expect_tx(&kv_full[s], nvc * 2 * DH * 2048);
      __syncwarp();
      const int c = min(lane / (2 * DH), 7), which = (lane / DH) & 1, dh = lane % DH;
      const int page = __shfl_sync(0xffffffffu, pg, c);
      if (lane < nbox) {
        if (c < nvc) {
          const int tok = tok_tile + c * 16;
          const bool bad = page < 0 || page >= p.num_pages;
          unsigned char *dst = smem + L::KV_OFF + s * L::STAGE_BYTES + which * L::K_BYTES +
                               dh * (kN * 128) + c * 16 * 128;
          // a bad page id loads from page 0 (in bounds) and is flagged; its
          // keys still count, so the result is wrong but nothing faults
          tma_load_4d(dst, &kvmap, dh * 64, h, tok % p.ps, (bad ? 0 : page) * 2 + which,
                      &kv_full[s], pol_kv);
          if (bad && which == 0 && dh == 0) flag(p.status, MI_STATUS_BAD_PAGE);
        }
      }
    }
    // no copy may be in flight when the CTA retires
    for (int j = max(0, n_tiles - 2); j < n_tiles; ++j)
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&kv_full[j & 1], (j >> 1) & 1))) ok = false;
  } else if (warp == 1) {
    // ============================ MMA issuer ================================
    if (lane == 0) {
      const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      const uint32_t idesc_qk = umma_idesc(fmt, false, kN, kM);
      const uint32_t idesc_pv = umma_idesc(fmt, true, D, kM);
      const uint32_t q_addr = smem_u32(smem + L::Q_OFF);
      const uint32_t p_addr = smem_u32(smem + L::P_OFF);
      // S = Q K_j^T for the K tile in stage j & 1
      auto issue_qk = [&](int j) {
        const uint32_t k_addr = smem_u32(smem + L::KV_OFF + (j & 1) * L::STAGE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kM * 128) + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * (kN * 128) + (kk & 3) * 32;
          umma(tmem_s, umma_desc(q_addr + off, 16, 1024), umma_desc(k_addr + koff, 16, 1024),
               idesc_qk, kk > 0);
        }
        umma_commit(s_full);
      };
      if (!mbar_wait_bounded(q_full, 0) || !mbar_wait_bounded(&kv_full[0], 0)) ok = false;
      if (ok) {
        tc_fence_after();
        issue_qk(0);
      }
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int s = j & 1;
        const uint32_t v_addr = smem_u32(smem + L::KV_OFF + s * L::STAGE_BYTES) + L::K_BYTES;
        if (j + 1 < n_tiles) {  // S_{j+1} once S_j is out of TMEM, under softmax j
          if (!mbar_wait_bounded(s_free, j & 1) ||
              !mbar_wait_bounded(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_qk(j + 1);
        }
        if (!mbar_wait_bounded(p_full, j & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kN / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * (kM * 128) + (kk & 3) * 32;
          // V: MN-major, 64-wide d blocks kN*128 bytes apart, 8-token groups 1 KB apart
          umma(tmem_o, umma_desc(p_addr + aoff, 16, 1024),
               umma_desc(v_addr + kk * 16 * 128, kN * 128, 1024), idesc_pv, (j > 0 || kk > 0));
        }
        umma_commit(&kv_empty[s]);
        umma_commit(o_done);
      }
      // the last products must land before TMEM is freed
      if (ok && !mbar_wait_bounded(o_done, (n_tiles - 1) & 1)) ok = false;
    }
    __syncwarp();
  } else {
    // ====================== softmax + epilogue (warps 2..5) =================
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // packed row == TMEM lane
    const int t = r / g, jh = r % g;
    const bool row_ok = r < m_used && t < rows_tok;
    int lim = p.causal ? lk - lq + t0 + t + 1 : lk;
    lim = min(lim, lk);
    if (!row_ok) lim = 0;
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    float m = -INFINITY, l = 0.f;
    unsigned char *prow = smem + L::P_OFF;
    for (int j = 0; j < n_tiles; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(s_full, j & 1))) { ok = false; break; }
      tc_fence_after();
      float sv[kN];
#pragma unroll
      for (int c = 0; c < kN / 32; ++c) tmem_ld32(tmem_s + lane_base + c * 32, sv + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      const int kbase = j * kN;
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < kN; ++c) {
        sv[c] = (kbase + c < lim) ? sv[c] * p.scale_log2 : -INFINITY;
        mt = fmaxf(mt, sv[c]);
      }
      const float m_new = fmaxf(m, mt);
      const float ms = m_new == -INFINITY ? 0.f : m_new;
      const float corr = m == m_new ? 1.f : exp2f(m - ms);
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < kN; ++c) {
        sv[c] = exp2f(sv[c] - ms);
        sum += sv[c];
      }
      l = l * corr + sum;
      m = m_new;
      // P_{j-1} must have been consumed (and O_{j-1} complete) before P_j / O
      if (j > 0) {
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(o_done, (j - 1) & 1))) { ok = false; break; }
        tc_fence_after();
      }
#pragma unroll
      for (int kb = 0; kb < kN / 64; ++kb) {
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const float *x = sv + kb * 64 + cc * 8;
          uint4 w;
          w.x = Pack2<T>::run(x[0], x[1]);
          w.y = Pack2<T>::run(x[2], x[3]);
          w.z = Pack2<T>::run(x[4], x[5]);
          w.w = Pack2<T>::run(x[6], x[7]);
          *reinterpret_cast<uint4 *>(prow + kb * (kM * 128) + swz(r, cc)) = w;
        }
      }
      if (j > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float ov[32];
          tmem_ld32(tmem_o + lane_base + c * 32, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= corr;
          tmem_st32(tmem_o + lane_base + c * 32, ov);
        }
        tmem_wait_st();
      }
      fence_proxy_async_smem();  // P visible to the tensor core
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // ---- epilogue -----------------------------------------------------------
    if (__all_sync(0xffffffffu, ok && mbar_wait_bounded(o_done, (n_tiles - 1) & 1))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T *o = static_cast<T *>(p.out) +
             (static_cast<int64_t>(q_start + t0 + t) * p.hq + h * g + jh) * D;
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
      if (row_ok && p.lse)
        p.lse[static_cast<int64_t>(q_start + t0 + t) * p.hq + h * g + jh] =
            l > 0.f ? (m + __log2f(l)) * kLn2 : -INFINITY;
    } else {
      ok = false;
    }
  }
  if (!ok && lane == 0) flag(p.status, MI_STATUS_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256)
                 : "memory");
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
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> (dev & 63) & 1ull)) {
    if (cudaFuncSetAttribute(prefill_tc_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             L::SMEM) != cudaSuccess)
      return check_launch("prefill_tc_kernel smem attribute");
    attr_set |= 1ull << (dev & 63);
  }
  // upper bound on (request, query tile) pairs: sum ceil(L_b / tq) <= total/tq + batch
  const int tiles = (p.total_q + tq - 1) / tq + p.batch;
  dim3 grid(tiles, p.hkv);
  prefill_tc_kernel<T, D><<<grid, kThreadsP, L::SMEM, s>>>(qmap, kvmap, p);
  return check_launch("prefill_tc_kernel");
}

}  // namespace

int launch_prefill_tc(const PrefillParams &p, int dtype, cudaStream_t s) {
  if (!(dtype == MI_DTYPE_BF16 || dtype == MI_DTYPE_F16)) return -1;
  if (!(p.d == 64 || p.d == 128)) return -1;
  if (p.group > kM || p.ps % 16 != 0 || p.ps > 256 || p.batch > kMaxBatchTc) return -1;
  if (p.hkv > 65535 || p.num_pages * 2 > (1LL << 31)) return -1;
  if (static_cast<int64_t>(p.total_q) + kM > (1LL << 31)) return -1;
  if (dtype == MI_DTYPE_BF16)
    return p.d == 128 ? launch_t<__nv_bfloat16, 128>(p, dtype, s)
                      : launch_t<__nv_bfloat16, 64>(p, dtype, s);
  return p.d == 128 ? launch_t<__half, 128>(p, dtype, s) : launch_t<__half, 64>(p, dtype, s);
}

}  // namespace mi
