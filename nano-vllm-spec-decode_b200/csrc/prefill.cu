// Varlen causal prefill attention for sm_100a (replaces flash_attn_varlen_func at nanovllm/layers/attention.py:67-70
// for query runs longer than the decode kernel's 48-row tile: prefill chunks, with or without a paged prefix).
//
// Work item = (128-row query tile of one sequence, q head).  A one-CTA plan kernel (also used by prefill_pair.cu,
// whose items are two tiles) lists the items heaviest first (most key tiles under the causal mask); persistent CTAs
// take the first wave by block index and every later item from an atomic counter (longest-processing-time-first
// list scheduling), so the long tiles start first and the short ones fill in wherever a CTA frees up.
//
// Per item: S = Q K^T with M = 128 query rows on the TMEM lanes, N = 128 keys (A = Q, B = K tile, both K-major
// 128B-swizzled straight from TMA); P = exp2(S * scale - m) in bf16, written back into its own S buffer in tensor
// memory (keys [0, 64) in columns [0, 32), keys [64, 128) in columns [64, 96): each key half's P lands in that
// half's own S columns); O += P V in TMEM (A = P read from TMEM, B = V tile, MN-major, straight from TMA).
// Keeping P out of shared memory pays for a 3-stage V ring.  Each query row is shared by two threads, one per
// key half (see the warp roles below).  O is rescaled in TMEM only when a row's maximum grows by more than 2^8
// (until then P values up to 256 are exact enough in bf16 and FP32 sums).
//
// Warp roles (384 threads): 0 = Q + K producer (also publishes the item descriptors), 3 = V producer, 1 = TMEM owner
// + UMMA issuer, 2 = output writer, 4..11 = softmax + epilogue in two warpgroups: thread (group w, row t) owns keys
// [64w, 64w + 64) of query row t, so each S tile costs a thread 64 exponentials (a quarter of them on the FMA pipe
// through exp2_poly2) and two warps share each SM quarter to hide MUFU / TMEM latency.  A thread first takes its
// weights against the row's running maximum; one named-barrier vote per tile tells whether any half-row sum reached
// 2^8 (a weight may have), and only then do the two halves of each row exchange their maxima through shared memory
// and redo the weights.  The row sums meet in spare TMEM columns.  The softmax warps stage
// the normalised O tile in the item's Q buffer (TMA's 128-byte-swizzled two-slab layout) and move on; the writer
// warp stores it (TMA for full 128-row tiles, plain stores for a sequence's last partial tile) and frees the buffer.
#include "nva_ptx.cuh"
#include "nva_kernels.h"

namespace nva {

namespace {

constexpr int kThreads = 384;           // 4 service warps + 2 softmax warpgroups
constexpr int kSlab = 128 * 128;       // 128 rows x 128 bytes
constexpr int kTile = 2 * kSlab;       // 128 rows x 256 bytes (all 128 dims, or 128 keys of P)
constexpr int kItemRing = 8;           // item descriptors: producer is at most ~5 items ahead of the softmax warps
constexpr float kNegInf = -__builtin_huge_valf();
constexpr uint32_t kFull = 0xffffffffu;
constexpr float kRescaleLog2 = 8.0f;   // rescale O only when a row maximum grows by more than this (log2 units)

// shared memory map (offsets from a 1024-aligned base)
constexpr int kKStages = 2;
constexpr int kVStages = 3;
constexpr int kOffQ = 0;                              // 2 x Q tile
constexpr int kOffK = kOffQ + 2 * kTile;              // K ring
constexpr int kOffV = kOffK + kKStages * kTile;       // V ring
constexpr int kOffBars = kOffV + kVStages * kTile;    // 32 x u64
constexpr int kOffItems = kOffBars + 32 * 8;      // kItemRing x 2 x int4
constexpr int kOffRed = kOffItems + kItemRing * 32;   // [2 tiles][2 groups][128 rows] half-row maxima
constexpr int kOffTmem = kOffRed + 2 * 2 * 128 * 4;
constexpr int kOffAbort = kOffTmem + 4;
constexpr int kSmemBytes = kOffAbort + 4;             // the dynamic shared memory base is 1024-aligned (checked)
static_assert(kSmemBytes <= 232448, "prefill shared memory budget");

enum {
  B_QFULL = 0, B_QEMPTY = 2, B_KFULL = 4, B_KEMPTY = 6, B_VFULL = 8, B_VEMPTY = 11, B_SFULL = 14, B_PFULL = 16,
  B_ODONE = 17, B_ITEM = 18,  // B_ITEM + kItemRing <= B_OSTAGED
  B_OSTAGED = 26              // 2: normalised O of the item staged in Q buffer 0 / 1
};

struct Item {
  int b, qt, h, nkv;   // sequence, query tile, q head, key tiles under the causal mask
  int n, L, q0, k0;    // query rows, keys, first query row, first key row (contiguous K/V only)
  int rows;            // valid query rows in this tile
  bool valid;
};

// Item k of a CTA's sequence: plan entry k / H, head k % H.
__device__ __forceinline__ Item load_item(const PrefillParams& p, int k, int total) {
  Item it;
  const int pidx = k / p.num_heads;
  it.valid = pidx < total;
  if (!it.valid) return it;
  const int e = p.plan[1 + pidx];
  it.b = e >> 12;
  it.qt = e & 0xfff;
  it.h = k - pidx * p.num_heads;
  it.q0 = __ldg(p.cu_q + it.b);
  it.n = __ldg(p.cu_q + it.b + 1) - it.q0;
  it.k0 = __ldg(p.cu_k + it.b);
  it.L = __ldg(p.cu_k + it.b + 1) - it.k0;
  it.rows = min(128, it.n - it.qt * 128);
  it.nkv = prefill_tile_nkv(it.n, it.L, it.qt);
  return it;
}

// ------------------------------------------------------------------------------------------------ plan kernel
// Work items of p.tiles_per_item consecutive 128-row query tiles (1 for prefill_kernel, 2 for prefill_pair_kernel).
// plan[0] = number of items of sequences with q_len >= min_q; plan[1 + i] = (seq << 12) | item of the sequence,
// ordered by descending key-tile count of the item's last tile (ties by position), so persistent CTAs start the
// longest items first.
__global__ void __launch_bounds__(1024) prefill_plan_kernel(const PrefillParams p) {
  __shared__ int cost[kMaxPrefillTiles];
  __shared__ int code[kMaxPrefillTiles];
  __shared__ int warp_tot[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // launched with a programmatic dependency: the preceding kernel (or the last call's prefill kernel, which may
  // still read the plan) completes before the plan is rewritten; then the call's next kernel may start its blocks
  griddep_wait();
  if (tid == 0) griddep_launch_dependents();
  // items per sequence and their exclusive prefix (B <= 1024: one element per thread)
  const int tpi = p.tiles_per_item;
  int nt = 0, n = 0, L = 0;
  if (tid < p.num_seqs) {
    const int a = p.cu_q[tid];
    n = p.cu_q[tid + 1] - a;
    L = p.cu_k[tid + 1] - p.cu_k[tid];
    nt = n >= p.min_q && n > 0 ? (n + 128 * tpi - 1) / (128 * tpi) : 0;
  }
  int x = nt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(kFull, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  int before = 0, total = 0;
  for (int w = 0; w < 32; ++w) {
    if (w < warp) before += warp_tot[w];
    total += warp_tot[w];
  }
  const int off = before + x - nt;
  const int cap = min(p.q_tiles_bound, kMaxPrefillTiles);
  total = min(total, cap);
  for (int u = 0; u < nt; ++u) {
    const int i = off + u;
    if (i < cap) {
      cost[i] = prefill_tile_nkv(n, L, min(tpi * u + tpi - 1, (n - 1) / 128));
      code[i] = (tid << 12) | u;
    }
  }
  __syncthreads();
  // rank by (cost desc, index asc); O(total^2 / 1024) comparisons
  for (int i = tid; i < total; i += 1024) {
    const int ci = cost[i];
    int rank = 0;
    for (int j = 0; j < total; ++j) {
      const int cj = cost[j];
      rank += (cj > ci) || (cj == ci && j < i);
    }
    p.plan[1 + rank] = code[i];
  }
  if (tid == 0) {
    p.plan[0] = total;
    p.plan[1 + p.q_tiles_bound] = 0;   // work counter of the main kernel
  }
}

// ------------------------------------------------------------------------------------------------ main kernel
__global__ void __launch_bounds__(kThreads, 1)
prefill_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
               const PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem_raw) & 1023u) != 0) {   // the swizzled layouts need a 1024-byte aligned base
    if (threadIdx.x == 0) atomicOr(&g_error_word, kErrTimeout);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  int4* items = reinterpret_cast<int4*>(smem + kOffItems);
  float* red = reinterpret_cast<float*>(smem + kOffRed);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + kOffAbort);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool paged = p.block_tables != nullptr;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_QFULL + i], 1);
      mbar_init(&bars[B_QEMPTY + i], 1);     // released by the writer warp once the staged O has been read
      mbar_init(&bars[B_OSTAGED + i], 256);  // the softmax threads' halves of O staged
      mbar_init(&bars[B_KFULL + i], 1);
      mbar_init(&bars[B_KEMPTY + i], 1);
      mbar_init(&bars[B_SFULL + i], 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(&bars[B_VFULL + i], 1);
      mbar_init(&bars[B_VEMPTY + i], 1);
    }
    mbar_init(&bars[B_PFULL], 256);
    mbar_init(&bars[B_ODONE], 1);
    for (int i = 0; i < kItemRing; ++i) mbar_init(&bars[B_ITEM + i], 1);
    *abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    if (p.o_tma) tma_prefetch_desc(&tm_o);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Launched with a programmatic dependency on the preceding kernel.  After the plan kernel (wait_primary) the plan
  // is read only once that grid has completed; after the decode kernel of the same call (which waited for the plan
  // kernel before letting this grid start) nothing here depends on it, and the blocks run beside its last blocks.
  if (p.wait_primary) griddep_wait();
  if (tid == 0) griddep_launch_dependents();
  const int total = p.plan[0];

  if (warp == 0 || warp == 3) {
    // ------------------------------------------------------------ Q+K (warp 0) and V (warp 3) producers
    const bool is_k = warp == 0;
    const CUtensorMap* tm = is_k ? &tm_k : &tm_v;
    uint8_t* ring = smem + (is_k ? kOffK : kOffV);
    uint64_t* full = bars + (is_k ? B_KFULL : B_VFULL);
    uint64_t* empty = bars + (is_k ? B_KEMPTY : B_VEMPTY);
    const int stages = is_k ? kKStages : kVStages;
    int g = 0;
    bool stop = false;
    int* counter = p.plan + 1 + p.q_tiles_bound;
    // The K producer takes each item and publishes it (nkv = 0: no more items) in the item ring; the V producer,
    // the UMMA issuer and the softmax warps follow the ring.  The ring cannot overrun: the K producer waits for the
    // Q buffer of item i - 2, whose epilogue comes after every consumer has read entry i - 2.
    for (int it_count = 0; !stop; ++it_count) {
      const int e = it_count % kItemRing;
      Item it;
      if (is_k) {
        int k = blockIdx.x;
        if (it_count > 0) {
          int v = 0;
          if (elect_one()) v = atomicAdd(counter, 1);
          k = gridDim.x + __reduce_add_sync(kFull, v);
        }
        it = load_item(p, k, total);   // invalid once k >= number of tiles x heads
        if (elect_one()) {
          items[2 * e] = it.valid ? make_int4(it.b, it.qt, it.h, it.nkv) : make_int4(0, 0, 0, 0);
          items[2 * e + 1] = it.valid ? make_int4(it.n, it.L, it.q0, it.rows) : make_int4(0, 0, 0, 0);
          mbar_arrive(&bars[B_ITEM + e]);
        }
        __syncwarp();
        if (!it.valid) break;
      } else {
        if (!mbar_wait_warp(&bars[B_ITEM + e], (it_count / kItemRing) & 1, abort)) break;
        const int4 i0 = items[2 * e];
        if (i0.w == 0) break;
        it.b = i0.x;
        it.h = i0.z;
        it.nkv = i0.w;
        it.k0 = paged ? 0 : __ldg(p.cu_k + it.b);
      }
      const int kvh = it.h / p.group;
      if (is_k) {
        const int qb = it_count & 1;
        if (!mbar_wait_warp(&bars[B_QEMPTY + qb], ((it_count >> 1) & 1) ^ 1, abort)) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(&bars[B_QFULL + qb], kTile);
          uint8_t* dst = smem + kOffQ + qb * kTile;
          tma_load_3d(dst, &tm_q, 0, it.h, it.q0 + it.qt * 128, &bars[B_QFULL + qb]);
          tma_load_3d(dst + kSlab, &tm_q, 64, it.h, it.q0 + it.qt * 128, &bars[B_QFULL + qb]);
        }
        __syncwarp();
      }
      for (int base = 0; base < it.nkv && !stop; base += 32) {
        // key-tile rows for the next 32 tiles (block-table reads in parallel across lanes)
        int row0 = 0;
        if (base + lane < it.nkv) {
          const int tok0 = (base + lane) * 128;
          if (paged) {
            int page = __ldg(p.block_tables + (int64_t)it.b * p.bt_stride + tok0 / p.block_size);
            if (page < 0 || page >= p.num_blocks) {
              if (is_k) atomicOr(&g_error_word, kErrBlockRange);
              page = -1;   // rows filled with zeros by TMA; nothing outside the pool is read
            }
            row0 = page * p.block_size + tok0 % p.block_size;
          } else {
            row0 = it.k0 + tok0;
          }
        }
        const int cnt = min(32, it.nkv - base);
        for (int i = 0; i < cnt; ++i, ++g) {
          const int r0 = __shfl_sync(kFull, row0, i);
          const int st = g % stages;
          if (!mbar_wait_warp(&empty[st], ((g / stages) & 1) ^ 1, abort)) {
            stop = true;
            break;
          }
          if (elect_one()) {
            mbar_arrive_expect_tx(&full[st], kTile);
            tma_load_3d(ring + st * kTile, tm, 0, kvh, r0, &full[st]);
            tma_load_3d(ring + st * kTile + kSlab, tm, 64, kvh, r0, &full[st]);
          }
          __syncwarp();
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    constexpr uint32_t idesc_qk = umma_idesc_bf16(128, 128, false, false);
    constexpr uint32_t idesc_pv = umma_idesc_bf16(128, 128, false, true);
    const uint32_t v_base = smem_u32(smem + kOffV);
    const uint64_t q_desc0 = umma_desc_sw128(smem_u32(smem + kOffQ), 16, 1024);
    const uint64_t k_desc0 = umma_desc_sw128(smem_u32(smem + kOffK), 16, 1024);
    const uint64_t v_desc0 = umma_desc_sw128(v_base, kSlab, 1024);
    // Issue order: QK(0), QK(1), then PV(g), QK(g+2), ...  QK(g+2) overwrites the S buffer that holds P(g), so it
    // must follow PV(g) (the tensor pipe runs one thread's products in issue order); every wait is a blocking,
    // hardware-suspended mbarrier wait.  Tile indices g run across the CTA's items.
    int it_q = 0, j_q = 0, nkv_q = 0, gq = 0;   // next S product
    int it_p = 0, j_p = 0, gp = 0;              // next PV product
    bool ok = true, q_done = false;             // q_done: the item ring's end marker was read (it_q items)
    auto issue_qk = [&]() {
      if (!ok || q_done) return;
      const int qb = it_q & 1;
      if (j_q == 0) {
        const int e = it_q % kItemRing;
        if (!mbar_wait_warp(&bars[B_ITEM + e], (it_q / kItemRing) & 1, abort)) { ok = false; return; }
        nkv_q = items[2 * e].w;
        if (nkv_q == 0) {
          q_done = true;
          return;
        }
        if (!mbar_wait_warp(&bars[B_QFULL + qb], (it_q >> 1) & 1, abort)) { ok = false; return; }
      }
      const int st = gq & 1;
      if (!mbar_wait_warp(&bars[B_KFULL + st], (gq >> 1) & 1, abort)) { ok = false; return; }
      tc_fence_after();
      if (elect_one()) {
        // K-major SW128 operands: step k sits at +32 B within a 128-byte row, steps 4..7 in the second slab
        constexpr uint32_t kOff[8] = {0, 2, 4, 6, kSlab >> 4, (kSlab >> 4) + 2, (kSlab >> 4) + 4, (kSlab >> 4) + 6};
        umma_bf16_ss_x8(tmem + st * 128, q_desc0 + ((qb * kTile) >> 4), k_desc0 + ((st * kTile) >> 4), idesc_qk, 0u,
                        kOff, kOff);
        umma_commit(&bars[B_SFULL + st]);
        umma_commit(&bars[B_KEMPTY + st]);
      }
      __syncwarp();
      ++gq;
      if (++j_q == nkv_q) {
        j_q = 0;
        ++it_q;
      }
    };
    issue_qk();
    issue_qk();
    // S runs two tiles ahead of PV, so the end marker is read before PV reaches the last item
    while (ok && (!q_done || it_p < it_q)) {
      const int nkv_p = items[2 * (it_p % kItemRing)].w;   // published (and awaited) before this item's first QK
      const int st = gp % kVStages;
      if (!mbar_wait_warp(&bars[B_PFULL], gp & 1, abort)) break;
      if (!mbar_wait_warp(&bars[B_VFULL + st], (gp / kVStages) & 1, abort)) break;
      tc_fence_after();
      if (elect_one()) {
        const uint64_t vd = v_desc0 + ((st * kTile) >> 4);
        const uint32_t pa = tmem + (gp & 1) * 128;   // P of tile gp: columns [0, 32) and [64, 96) of its S buffer
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)   // V: 16 keys (2048 B) per step; P: 8 columns per step; fresh O per item
          umma_bf16_ts(tmem + 256, pa + kk * 8 + (kk >= 4 ? 32 : 0), vd + kk * (2048 >> 4), idesc_pv,
                       (j_p > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bars[B_ODONE]);
        umma_commit(&bars[B_VEMPTY + st]);
      }
      __syncwarp();
      ++gp;
      if (++j_p == nkv_p) {
        j_p = 0;
        ++it_p;
      }
      issue_qk();
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ output writer
    for (int it_count = 0;; ++it_count) {
      const int e = it_count % kItemRing;
      if (!mbar_wait_warp(&bars[B_ITEM + e], (it_count / kItemRing) & 1, abort)) break;
      const int4 i0 = items[2 * e], i1 = items[2 * e + 1];
      if (i0.w == 0) break;
      const int qb = it_count & 1;
      if (!mbar_wait_warp(&bars[B_OSTAGED + qb], (it_count >> 1) & 1, abort)) break;
      const int h = i0.z, row0 = i1.z + i0.y * 128, rows = i1.w;
      const uint8_t* stage = smem + kOffQ + qb * kTile;
      if (p.o_tma && rows == 128) {
        if (elect_one()) {
          tma_store_3d(&tm_o, stage, 0, h, row0);
          tma_store_3d(&tm_o, stage + kSlab, 64, h, row0);
          tma_store_commit_wait_read();
          mbar_arrive(&bars[B_QEMPTY + qb]);
        }
        __syncwarp();
      } else {
        // lane: 8 bytes (dims 4 lane .. 4 lane + 3) of each row, i.e. 16-byte chunk lane / 2 of the 256-byte row
        const int chunk = lane >> 1;
        const int off = (chunk >> 3) * kSlab + ((lane & 1) << 3);
#pragma unroll 1
        for (int r0 = 0; r0 < rows; r0 += 8) {
          uint2 v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = r0 + i;
            v[i] = *reinterpret_cast<const uint2*>(stage + off + r * 128 + (((chunk & 7) ^ (r & 7)) << 4));
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = r0 + i;
            if (r < rows)
              *reinterpret_cast<uint2*>(p.out + (int64_t)(row0 + r) * p.out_row_stride + (int64_t)h * kHeadDim +
                                        lane * 4) = v[i];
          }
        }
        fence_proxy_async_smem();   // these generic reads before the next TMA write into the buffer
        __syncwarp();
        if (elect_one()) mbar_arrive(&bars[B_QEMPTY + qb]);
      }
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");   // every TMA store of this warp complete
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue: two warpgroups
    // All eight softmax warps run the same sequence of named barriers (bar.red.or of "gave up"), one per tile and
    // two per item, so they always leave together if a wait expires.
    const int wg = (warp - 4) >> 2;           // key half: columns [64 wg, 64 wg + 64)
    const int wq = warp & 3;                  // TMEM lane quadrant
    const int t = wq * 32 + lane;             // query row within the tile
    const int c0 = 64 * wg;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    int g = 0, pv_seen = 0, it_count = 0;
    bool alive = true;
    for (;; ++it_count) {
      const int e = it_count % kItemRing;
      alive = alive && mbar_wait_warp(&bars[B_ITEM + e], (it_count / kItemRing) & 1, abort);
      int4 i0 = make_int4(0, 0, 0, 1), i1 = make_int4(0, 0, 0, 0);
      if (alive) {
        i0 = items[2 * e];
        i1 = items[2 * e + 1];
      }
      if (named_bar_any(1, 256, !alive || i0.w == 0)) break;   // end marker (or a wait gave up): all leave
      const int nkv = i0.w, n = i1.x, L = i1.y, qt = i0.y;
      const int lim = L - n + qt * 128 + t;   // this row sees keys <= lim
      float m_used = kNegInf, l = 0.f;       // l: this thread's half of the row sum
      for (int j = 0; j < nkv; ++j, ++g) {
        const int st = g & 1;              // S / P buffer
        const int vs = g % kVStages;       // V ring slot
        float s[64];
        float mpart = kNegInf;
        // paged keys past the sequence end may be stale or uninitialised: zero V there (P is 0 there anyway)
        if (alive && wg == 0 && paged && j * 128 + 127 >= L) {
          alive = mbar_wait_warp(&bars[B_VFULL + vs], (g / kVStages) & 1, abort);
          if (alive && j * 128 + t >= L) {
            uint8_t* vrow = smem + kOffV + vs * kTile + t * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0u, 0u, 0u, 0u);
              *reinterpret_cast<uint4*>(vrow + kSlab + c * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
            // generic-proxy writes, read by the PV product through the async proxy: ordered by this fence and this
            // thread's later PFULL arrival
            fence_proxy_async_smem();
          }
        }
        alive = alive && mbar_wait_warp(&bars[B_SFULL + st], (g >> 1) & 1, abort);
        const int kmax = lim - j * 128 - c0;     // columns > kmax of this half are masked for this row
        // Weights against the running maximum (the same value in both halves of a row).  A half-row sum below 2^8
        // shows that no weight reached 2^8, i.e. the row maximum did not grow past the rescale threshold on this
        // half.  One vote per tile (the named barrier the maximum exchange used): when no thread needs more, the
        // tile is done without its maximum; otherwise all take the exact path (maximum, exchange, rescale, weights
        // again).  Masked keys hold -inf, so their MUFU weights are exp2(-inf) = 0; a row that has seen no key yet
        // (m_used = -inf) subtracts 0 and gets only zeros.
        float pk[32];
        float hsum = 0.f;
        auto weights = [&]() {
          const float neg_m = m_used == kNegInf ? 0.f : -m_used;
          const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(neg_m, neg_m);
          float2 sum4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                            make_float2(0.f, 0.f)};
          const bool full = kmax >= 63;
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            const float2 x = ffma2(make_float2(s[c], s[c + 1]), sc2, nm2);
            float2 pp;
            if ((c & 7) == 6) {   // a quarter of the exponentials on the FMA pipe (2^-126 at -inf: zero them)
              pp = exp2_poly2(x);
              if (!full) {
                pp.x = c <= kmax ? pp.x : 0.f;
                pp.y = c + 1 <= kmax ? pp.y : 0.f;
              }
            } else {
              pp = make_float2(fast_exp2(x.x), fast_exp2(x.y));
            }
            sum4[(c >> 1) & 3] = fadd2(sum4[(c >> 1) & 3], pp);
            pk[c >> 1] = __uint_as_float(pack_bf16x2(pp.x, pp.y));
          }
          const float2 s01 = fadd2(fadd2(sum4[0], sum4[1]), fadd2(sum4[2], sum4[3]));
          hsum = s01.x + s01.y;
        };
        bool exact = true;
        if (alive) {
          tc_fence_after();
          tmem_ld64(t_lane + st * 128 + c0, s);
          if (kmax < 63) {
#pragma unroll
            for (int c = 0; c < 64; ++c) s[c] = c <= kmax ? s[c] : kNegInf;
          }
          if (m_used != kNegInf) {
            weights();
            exact = !(hsum < 256.f);
            // P (bf16 pairs, lower half = even key): keys [64 wg, 64 wg + 64) -> columns [64 wg, 64 wg + 32), this
            // group's own S columns (already in registers), so it may land before the other group has read its half
            tmem_st32_nowait(t_lane + st * 128 + 64 * wg, pk);
          }
        }
        if (named_bar_any(1, 256, !alive || exact)) {
          if (named_bar_any(1, 256, !alive)) {
            alive = false;
            break;
          }
          float m8[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            m8[i] = fmaxf(fmax3(fmax3(s[i], s[i + 8], s[i + 16]), s[i + 24], s[i + 32]),
                          fmax3(s[i + 40], s[i + 48], s[i + 56]));
          mpart = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
          red[(st * 2 + wg) * 128 + t] = mpart;
          named_bar_sync(1, 256);
          const float mx = fmaxf(mpart, red[(st * 2 + (wg ^ 1)) * 128 + t]);
          const float m_cand = fmaxf(m_used, mx * p.scale_log2);
          const bool rescale = m_used != kNegInf && m_cand > m_used + kRescaleLog2;
          if (j > 0 && __any_sync(kFull, rescale)) {
            // O must hold every earlier PV product of this item before it is rescaled
            if (pv_seen < g) {
              alive = mbar_wait_warp(&bars[B_ODONE], (g - 1) & 1, abort);
              pv_seen = g;
            }
            if (alive) {
              const float alpha = rescale ? fast_exp2(m_used - m_cand) : 1.f;
              tc_fence_after();
#pragma unroll 1
              for (int c = 0; c < 64; c += 32) {
                float ot[32];
                tmem_ld32(t_lane + 256 + c0 + c, ot);
#pragma unroll
                for (int i = 0; i < 32; ++i) ot[i] *= alpha;
                tmem_st32(t_lane + 256 + c0 + c, ot);
              }
              if (rescale) l *= alpha;
            }
          }
          if (rescale || m_used == kNegInf) m_used = m_cand;
          weights();
          tmem_wait_st();   // the fast path's store of these columns (if any) lands first
          tmem_st32_nowait(t_lane + st * 128 + 64 * wg, pk);
        }
        if (alive) {
          tmem_wait_st();   // this group's P stores (above) complete
          l += hsum;
          // Observe PV(g-1) before handing over P(g), so that at most one PV product is ever unobserved: otherwise
          // P(g+1) could complete the PFULL phase after P(g) before the issuer saw P(g)'s (its parity wait would
          // then wait for a phase that needs PV(g) itself), and PV(g) could complete ODONE before this wait for
          // PV(g-1) (the same two-phase aliasing).
          if (pv_seen < g) {
            alive = mbar_wait_warp(&bars[B_ODONE], (g - 1) & 1, abort);
            pv_seen = g;
          }
          tc_fence_before();
          if (alive) mbar_arrive(&bars[B_PFULL]);
        }
      }
      // ---- epilogue: O / l.  The two half-row sums meet in TMEM columns 384/385; O is staged in the item's idle
      // Q buffer (its last S product ran before the last PV product) in TMA's layout: dims [0, 64) and [64, 128) in
      // two 128-row slabs, 16-byte chunk k of row r at slot k ^ (r & 7); the writer warp takes it from there.
      if (alive) {
        alive = mbar_wait_warp(&bars[B_ODONE], (g - 1) & 1, abort);
        pv_seen = g;
        if (alive) {
          tmem_st1(t_lane + 384 + wg, l);
          tc_fence_before();
        }
      }
      if (named_bar_any(1, 256, !alive)) break;
      tc_fence_after();
      float lp[2];
      tmem_ld2(t_lane + 384, lp);
      const float lt = lp[0] + lp[1];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const int qb = it_count & 1;
      uint8_t* stage = smem + kOffQ + qb * kTile;
#pragma unroll 1
      for (int c = 0; c < 64; c += 32) {
        float ot[32];
        tmem_ld32(t_lane + 256 + c0 + c, ot);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 v;
          v.x = pack_bf16x2(ot[i] * inv, ot[i + 1] * inv);
          v.y = pack_bf16x2(ot[i + 2] * inv, ot[i + 3] * inv);
          v.z = pack_bf16x2(ot[i + 4] * inv, ot[i + 5] * inv);
          v.w = pack_bf16x2(ot[i + 6] * inv, ot[i + 7] * inv);
          const int chunk = (c0 + c + i) >> 3;   // 16-byte chunk of the 256-byte row
          *reinterpret_cast<uint4*>(stage + (chunk >> 3) * kSlab + t * 128 + (((chunk & 7) ^ (t & 7)) << 4)) = v;
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();   // staged rows visible to the writer's TMA store
      mbar_arrive(&bars[B_OSTAGED + qb]);
    }
  }

  __syncthreads();
  if (*abort) {
    if (tid == 0) atomicOr(&g_error_word, kErrTimeout);
    for (int i = 0; i < 1000; ++i) sleep_ns(1000);
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  // the grid completes only after the preceding one has (a later grid that waits for this one can rely on both)
  griddep_wait();
}

}  // namespace

cudaError_t launch_prefill_plan(const PrefillParams& p, cudaStream_t stream) {
  if (p.num_seqs > kMaxDecodeSeqs || p.q_tiles_bound > kMaxPrefillTiles) return cudaErrorInvalidValue;
  return launch_kernel(prefill_plan_kernel, dim3(1), dim3(1024), 0, stream, true, p);
}

cudaError_t launch_prefill(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                           const CUtensorMap& tm_o, const PrefillParams& p, int grid, cudaStream_t stream) {
  if (p.num_seqs > kMaxDecodeSeqs || p.q_tiles_bound > kMaxPrefillTiles) return cudaErrorInvalidValue;
  const cudaError_t e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  return launch_kernel(prefill_kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, true, tm_q, tm_k, tm_v, tm_o,
                       p);
}

}  // namespace nva
