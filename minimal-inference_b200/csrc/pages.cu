// Kernel (4): device-side page pool, slot page tables and step metadata.
//
// Replaces PagedKVCache's Python free list (scheduler.py:168-221), the page
// growth and CSR building of a decode step (scheduler.py:842-879), the
// graph-bucket padding of that metadata (scheduler.py:881-902) and the
// per-page, per-layer zero_() launches of release (scheduler.py:216-221).
// Everything runs on the device from caller-owned buffers, so a decode step
// (growth included) can live inside a CUDA graph.
//
// Pool state: free_ring[num_pages] (a FIFO ring of free page ids) and
// pool_ctrl[4] = {head, free_count, reserved, reserved}. The ring starts as
// 0..num_pages-2 in order; page num_pages-1 is the scratch page and never
// enters it. Pops take from the head, releases append at the tail, exactly
// as the reference's deque(popleft/append), so page tables match it.
//
// The pool kernels are single-CTA (sequential FIFO semantics); the zeroing
// kernel spreads (page, layer) pairs over the grid with 16-byte stores.
#include "mi_common.cuh"

namespace mi {
namespace {

constexpr int kPoolThreads = 1024;

// Block-wide exclusive scan of one int per thread (blockDim.x == 1024).
__device__ int block_excl_scan(int v, int *s_warp, int &total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < (blockDim.x >> 5) ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;  // inclusive warp prefix
  }
  __syncthreads();
  total = s_warp[(blockDim.x >> 5) - 1];
  const int before = warp ? s_warp[warp - 1] : 0;
  __syncthreads();
  return before + x - v;
}

__global__ void pool_init_kernel(int32_t *ring, int32_t *ctrl, int num_pages) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < num_pages; i += gridDim.x * blockDim.x)
    ring[i] = i < num_pages - 1 ? i : -1;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    ctrl[0] = 0;
    ctrl[1] = num_pages - 1;
    ctrl[2] = 0;
    ctrl[3] = 0;
  }
}

// Pop sum(counts) pages into out[0..total), FIFO.
__global__ void __launch_bounds__(kPoolThreads) page_alloc_kernel(
    int32_t *ring, int32_t *ctrl, int num_pages, const int32_t *counts, int n, int32_t *out,
    int32_t *status) {
  __shared__ int s_total;
  if (threadIdx.x == 0) s_total = 0;
  __syncthreads();
  int local = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) local += max(counts[i], 0);
  local = __reduce_add_sync(0xffffffffu, local);
  if ((threadIdx.x & 31) == 0 && local) atomicAdd(&s_total, local);
  __syncthreads();
  const int total = s_total;
  const int head = ctrl[0], free_count = ctrl[1];
  if (total > free_count) {
    for (int k = threadIdx.x; k < total; k += blockDim.x) out[k] = -1;
    if (threadIdx.x == 0) flag(status, MI_STATUS_OUT_OF_PAGES);
    return;
  }
  for (int k = threadIdx.x; k < total; k += blockDim.x) out[k] = ring[(head + k) % num_pages];
  __syncthreads();
  if (threadIdx.x == 0) {
    ctrl[0] = (head + total) % num_pages;
    ctrl[1] = free_count - total;
  }
}

// Zero every layer's copy of pages[i] (grid: (n, layers)); block (0, 0) also
// appends the pages to the ring tail when `push`.
__global__ void __launch_bounds__(256) page_release_kernel(
    int32_t *ring, int32_t *ctrl, int num_pages, const int32_t *pages, int n,
    void *const *layers, int64_t page_bytes, int push, int32_t *status) {
  const int i = blockIdx.x;
  const int page = pages[i];
  if (page_bytes > 0 && page >= 0 && page < num_pages) {
    uint4 *dst = reinterpret_cast<uint4 *>(static_cast<unsigned char *>(layers[blockIdx.y]) +
                                           static_cast<int64_t>(page) * page_bytes);
    const int64_t nvec = page_bytes / 16;
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int64_t k = threadIdx.x; k < nvec; k += blockDim.x) dst[k] = z;
  } else if ((page < 0 || page >= num_pages) && threadIdx.x == 0 && blockIdx.y == 0) {
    flag(status, MI_STATUS_BAD_PAGE);
  }
  if (push && blockIdx.x == 0 && blockIdx.y == 0) {
    const int head = ctrl[0], free_count = ctrl[1];
    if (free_count + n > num_pages - 1) {
      if (threadIdx.x == 0) flag(status, MI_STATUS_POOL_OVERFLOW);
      return;
    }
    for (int k = threadIdx.x; k < n; k += blockDim.x)
      ring[(head + free_count + k) % num_pages] = pages[k];
    __syncthreads();
    if (threadIdx.x == 0) ctrl[1] = free_count + n;
  }
}

// Admission: pop counts[i] pages into slot slots[i]'s page-table row.
__global__ void __launch_bounds__(kPoolThreads) slot_alloc_kernel(
    int32_t *ring, int32_t *ctrl, int num_pages, int32_t *table, int32_t *nump, int max_slots,
    int maxp, const int32_t *slots, const int32_t *counts, int n, int32_t *status) {
  __shared__ int s_warp[32];
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  const int head = ctrl[0], free_count = ctrl[1];
  int carry = 0;
  // pass 1: validate (all or nothing)
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    int c = 0;
    if (i < n) {
      c = max(counts[i], 0);
      const int s = slots[i];
      if (s < 0 || s >= max_slots) atomicOr(&s_bad, MI_STATUS_BAD_BATCH_INDEX);
      else if (nump[s] + c > maxp) atomicOr(&s_bad, MI_STATUS_SLOT_FULL);
    }
    int tot;
    block_excl_scan(c, s_warp, tot);
    carry += tot;
  }
  if (carry > free_count) {
    if (threadIdx.x == 0) s_bad |= MI_STATUS_OUT_OF_PAGES;
  }
  __syncthreads();
  if (s_bad) {
    if (threadIdx.x == 0) flag(status, s_bad);
    return;
  }
  // pass 2: pop in request order
  carry = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int c = i < n ? max(counts[i], 0) : 0;
    int tot;
    const int off = carry + block_excl_scan(c, s_warp, tot);
    if (i < n) {
      const int s = slots[i];
      const int have = nump[s];
      for (int j = 0; j < c; ++j)
        table[static_cast<int64_t>(s) * maxp + have + j] = ring[(head + off + j) % num_pages];
      nump[s] = have + c;
    }
    carry += tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ctrl[0] = (head + carry) % num_pages;
    ctrl[1] = free_count - carry;
  }
}

// Retire, part 1: zero every page of the listed slots in every layer.
// grid: (n * maxp, layers); block (i*maxp + j, l) zeroes page j of slot i.
__global__ void __launch_bounds__(256) slot_zero_kernel(
    const int32_t *table, const int32_t *nump, int max_slots, int maxp, const int32_t *slots,
    int n, int num_pages, void *const *layers, int64_t page_bytes) {
  const int i = blockIdx.x / maxp, j = blockIdx.x % maxp;
  const int s = slots[i];
  if (s < 0 || s >= max_slots || j >= nump[s]) return;
  const int page = table[static_cast<int64_t>(s) * maxp + j];
  if (page < 0 || page >= num_pages) return;
  uint4 *dst = reinterpret_cast<uint4 *>(static_cast<unsigned char *>(layers[blockIdx.y]) +
                                         static_cast<int64_t>(page) * page_bytes);
  const int64_t nvec = page_bytes / 16;
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int64_t k = threadIdx.x; k < nvec; k += blockDim.x) dst[k] = z;
}

// Retire, part 2: append the slots' pages to the ring tail (slot order, then
// allocation order) and empty the slots.
__global__ void __launch_bounds__(kPoolThreads) slot_free_kernel(
    int32_t *ring, int32_t *ctrl, int num_pages, int32_t *table, int32_t *nump, int max_slots,
    int maxp, const int32_t *slots, int n, int32_t *status) {
  __shared__ int s_warp[32];
  const int head = ctrl[0], free_count = ctrl[1];
  auto valid = [&](int s) { return s >= 0 && s < max_slots; };
  int carry = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    if (i < n && !valid(slots[i])) flag(status, MI_STATUS_BAD_BATCH_INDEX);
    const int c = (i < n && valid(slots[i])) ? nump[slots[i]] : 0;
    int tot;
    block_excl_scan(c, s_warp, tot);
    carry += tot;
  }
  if (free_count + carry > num_pages - 1) {
    if (threadIdx.x == 0) flag(status, MI_STATUS_POOL_OVERFLOW);
    return;
  }
  int done = 0;
  for (int base = 0; base < n; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int s = (i < n && valid(slots[i])) ? slots[i] : -1;
    const int c = s >= 0 ? nump[s] : 0;
    int tot;
    const int off = done + block_excl_scan(c, s_warp, tot);
    for (int j = 0; j < c; ++j)
      ring[(head + free_count + off + j) % num_pages] = table[static_cast<int64_t>(s) * maxp + j];
    done += tot;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (valid(slots[i])) nump[slots[i]] = 0;
  if (threadIdx.x == 0) ctrl[1] = free_count + done;
}

// One step's metadata: page growth (lanes in order) + CSR of all lanes.
__global__ void __launch_bounds__(kPoolThreads) step_prepare_kernel(
    int32_t *ring, int32_t *ctrl, int num_pages, int32_t *table, int32_t *nump, int max_slots,
    int maxp, const int32_t *lane_slots, const int32_t *lane_pos, int lanes, int ps, int grow,
    int32_t *indptr, int32_t *indices, int cap, int32_t *last, int32_t *apos, int32_t *status) {
  __shared__ int s_warp[32];
  __shared__ int s_indptr[kPoolThreads + 1];
  __shared__ int s_flag;
  const int i = threadIdx.x;
  if (i == 0) s_flag = 0;
  __syncthreads();
  int slot = i < lanes ? lane_slots[i] : -1;
  if (slot >= max_slots) {
    atomicOr(&s_flag, MI_STATUS_BAD_BATCH_INDEX);
    slot = -1;
  }
  int pos = i < lanes ? lane_pos[i] : 0;
  if (slot >= 0 && pos < 0) {
    atomicOr(&s_flag, MI_STATUS_BAD_POSITION);
    slot = -1;
  }
  const int have = slot >= 0 ? nump[slot] : 0;
  int need = 0;
  if (slot >= 0 && grow) {
    need = max(0, cdiv(pos + 1, ps) - have);
    if (have + need > maxp) {
      atomicOr(&s_flag, MI_STATUS_SLOT_FULL);
      need = 0;
    }
  }
  int total_need;
  const int off = block_excl_scan(need, s_warp, total_need);
  const int head = ctrl[0], free_count = ctrl[1];
  const bool can_grow = total_need <= free_count;
  if (!can_grow && i == 0) atomicOr(&s_flag, MI_STATUS_OUT_OF_PAGES);
  int np = have;
  if (can_grow && need > 0) {
    for (int j = 0; j < need; ++j)
      table[static_cast<int64_t>(slot) * maxp + have + j] = ring[(head + off + j) % num_pages];
    np = have + need;
    nump[slot] = np;
  }
  __syncthreads();
  if (i == 0 && can_grow && total_need > 0) {
    ctrl[0] = (head + total_need) % num_pages;
    ctrl[1] = free_count - total_need;
  }
  // CSR over all lanes
  int total_pages;
  const int start = block_excl_scan(slot >= 0 ? np : 0, s_warp, total_pages);
  if (i < lanes) {
    s_indptr[i] = start;
    indptr[i] = start;
    int ll = 1;
    if (slot >= 0) {
      ll = (pos + 1) % ps;
      if (ll == 0) ll = ps;
    }
    last[i] = ll;
    apos[i] = slot >= 0 ? pos : 0;
  }
  if (i == 0) {
    indptr[lanes] = total_pages;
    s_indptr[lanes] = total_pages;
    if (total_pages > cap) atomicOr(&s_flag, MI_STATUS_SLOT_FULL);
  }
  __syncthreads();
  if (total_pages <= cap) {
    for (int l = 0; l < lanes; ++l) {
      const int s = lane_slots[l];
      if (s < 0 || s >= max_slots) continue;
      const int b0 = s_indptr[l], cnt = s_indptr[l + 1] - b0;
      for (int j = i; j < cnt; j += blockDim.x)
        indices[b0 + j] = table[static_cast<int64_t>(s) * maxp + j];
    }
  }
  if (i == 0 && s_flag) flag(status, s_flag);
}

}  // namespace
}  // namespace mi

using mi::fail;

extern "C" int mi_page_pool_init(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                                 mi_stream_t stream) {
  MI_REQUIRE(free_ring && pool_ctrl && num_pages >= 2, "pool_init: bad arguments");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int blocks = (num_pages + 1023) / 1024;
  mi::pool_init_kernel<<<blocks < 1024 ? blocks : 1024, 1024, 0, s>>>(free_ring, pool_ctrl,
                                                                       num_pages);
  return mi::check_launch("pool_init_kernel");
}

extern "C" int mi_page_alloc(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                             const int32_t *counts, int32_t n, int32_t *out_pages,
                             int32_t *status, mi_stream_t stream) {
  MI_REQUIRE(free_ring && pool_ctrl && num_pages >= 2 && n >= 0, "page_alloc: bad arguments");
  if (n == 0) return MI_OK;
  MI_REQUIRE(counts && out_pages, "page_alloc: null counts/out_pages");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  mi::page_alloc_kernel<<<1, mi::kPoolThreads, 0, s>>>(free_ring, pool_ctrl, num_pages, counts,
                                                        n, out_pages, status);
  return mi::check_launch("page_alloc_kernel");
}

extern "C" int mi_page_release(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                               const int32_t *pages, int32_t n, void *const *layer_pools,
                               int32_t num_layers, int64_t page_bytes, int32_t *status,
                               mi_stream_t stream) {
  MI_REQUIRE(free_ring && pool_ctrl && num_pages >= 2 && n >= 0, "page_release: bad arguments");
  if (n == 0) return MI_OK;
  MI_REQUIRE(pages && (num_layers == 0 || layer_pools), "page_release: null pages/layer_pools");
  MI_REQUIRE(page_bytes > 0 && page_bytes % 16 == 0, "page_release: page_bytes %lld not a multiple of 16",
             (long long)page_bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(n, num_layers > 0 ? num_layers : 1);
  mi::page_release_kernel<<<grid, 256, 0, s>>>(free_ring, pool_ctrl, num_pages, pages, n,
                                                 layer_pools, num_layers > 0 ? page_bytes : 0, 1,
                                                 status);
  return mi::check_launch("page_release_kernel");
}

extern "C" int mi_slot_alloc(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                             int32_t *page_table, int32_t *slot_num_pages, int32_t max_slots,
                             int32_t max_pages_per_slot, const int32_t *slots,
                             const int32_t *counts, int32_t n, int32_t *status,
                             mi_stream_t stream) {
  MI_REQUIRE(free_ring && pool_ctrl && page_table && slot_num_pages && num_pages >= 2 &&
                 max_slots > 0 && max_pages_per_slot > 0 && n >= 0,
             "slot_alloc: bad arguments");
  if (n == 0) return MI_OK;
  MI_REQUIRE(slots && counts, "slot_alloc: null slots/counts");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  mi::slot_alloc_kernel<<<1, mi::kPoolThreads, 0, s>>>(free_ring, pool_ctrl, num_pages,
                                                        page_table, slot_num_pages, max_slots,
                                                        max_pages_per_slot, slots, counts, n,
                                                        status);
  return mi::check_launch("slot_alloc_kernel");
}

extern "C" int mi_slot_release(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                               int32_t *page_table, int32_t *slot_num_pages, int32_t max_slots,
                               int32_t max_pages_per_slot, const int32_t *slots, int32_t n,
                               void *const *layer_pools, int32_t num_layers, int64_t page_bytes,
                               int32_t *status, mi_stream_t stream) {
  MI_REQUIRE(free_ring && pool_ctrl && page_table && slot_num_pages && num_pages >= 2 &&
                 max_slots > 0 && max_pages_per_slot > 0 && n >= 0,
             "slot_release: bad arguments");
  if (n == 0) return MI_OK;
  MI_REQUIRE(slots, "slot_release: null slots");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (num_layers > 0) {
    MI_REQUIRE(layer_pools && page_bytes > 0 && page_bytes % 16 == 0,
               "slot_release: bad layer_pools/page_bytes");
    const long long blocks = static_cast<long long>(n) * max_pages_per_slot;
    MI_REQUIRE(blocks < (1LL << 31), "slot_release: too many pages");
    dim3 grid(static_cast<unsigned>(blocks), num_layers);
    mi::slot_zero_kernel<<<grid, 256, 0, s>>>(page_table, slot_num_pages, max_slots,
                                                max_pages_per_slot, slots, n, num_pages,
                                                layer_pools, page_bytes);
    int rc = mi::check_launch("slot_zero_kernel");
    if (rc) return rc;
  }
  mi::slot_free_kernel<<<1, mi::kPoolThreads, 0, s>>>(free_ring, pool_ctrl, num_pages,
                                                       page_table, slot_num_pages, max_slots,
                                                       max_pages_per_slot, slots, n, status);
  return mi::check_launch("slot_free_kernel");
}

extern "C" int mi_step_prepare(int32_t *free_ring, int32_t *pool_ctrl, int32_t num_pages,
                               int32_t *page_table, int32_t *slot_num_pages, int32_t max_slots,
                               int32_t max_pages_per_slot, const int32_t *lane_slots,
                               const int32_t *lane_positions, int32_t num_lanes,
                               int32_t page_size, int32_t grow, int32_t *kv_indptr,
                               int32_t *kv_indices, int32_t indices_capacity,
                               int32_t *kv_last_page_len, int32_t *append_positions,
                               int32_t *status, mi_stream_t stream) {
  MI_REQUIRE(free_ring && pool_ctrl && page_table && slot_num_pages && lane_slots &&
                 lane_positions && kv_indptr && kv_indices && kv_last_page_len &&
                 append_positions,
             "step_prepare: null pointer argument");
  MI_REQUIRE(num_lanes >= 1 && num_lanes <= mi::kPoolThreads,
             "step_prepare: num_lanes %d outside [1, %d]", num_lanes, mi::kPoolThreads);
  MI_REQUIRE(page_size > 0 && max_slots > 0 && max_pages_per_slot > 0 && num_pages >= 2,
             "step_prepare: bad geometry");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  mi::step_prepare_kernel<<<1, mi::kPoolThreads, 0, s>>>(
      free_ring, pool_ctrl, num_pages, page_table, slot_num_pages, max_slots, max_pages_per_slot,
      lane_slots, lane_positions, num_lanes, page_size, grow, kv_indptr, kv_indices,
      indices_capacity, kv_last_page_len, append_positions, status);
  return mi::check_launch("step_prepare_kernel");
}
