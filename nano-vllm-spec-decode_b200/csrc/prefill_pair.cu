// Varlen causal prefill attention for sm_100a, work items of two query tiles: the variant of prefill.cu that the C
// ABI launches when a call carries enough query rows x heads to give every SM several such items (the pairing
// halves the number of items, so on small calls the single-tile kernel balances better).  Same plan kernel (with
// tiles_per_item = 2), same launch contract, same results up to the order of the FP32 additions.
//
// Work item = (two consecutive 128-row query tiles of one sequence, q head), heaviest first, persistent CTAs taking
// later items from an atomic counter as in prefill.cu.  Per item and key tile j, for each query tile w of the pair:
// S_w = Q_w K_j^T with M = 128 query rows on the TMEM lanes, N = 128 keys (A = Q_w, B = K tile, both K-major
// 128B-swizzled straight from TMA); P_w = exp2(S_w * scale - m) in bf16, written back into the first 64 columns of
// S_w in tensor memory; O_w += P_w V_j in TMEM (A = P_w read from TMEM, B = V tile, MN-major, straight from TMA).
// The two query tiles share every K and V tile.  TMEM (512 columns): S_0, S_1, O_0, O_1.  O is rescaled in TMEM only
// when a row's maximum grows by more than 2^8 (until then P values up to 256 are exact enough in bf16 and FP32
// sums).
//
// Warp roles (384 threads): 0 = Q + K producer (also publishes the item descriptors), 3 = V producer, 1 = TMEM owner
// + UMMA issuer, 2 idle, 4..7 and 8..11 = softmax + epilogue, one warpgroup per query tile: thread t of group w owns
// query row t of tile w whole (128 exponentials per key tile on the MUFU pipe; maximum and sum thread-local, so the
// groups never wait for each other), as two online-softmax steps of 64 keys each: one TMEM load per half, and a P
// store that completes in the background while the second half loads.  A half first takes its weights against the
// running maximum; only when a weight may have reached 2^8 (its half-row sum did) does it compute its own maximum
// and redo them.  The issuer interleaves the two tiles' products, so one group's softmax runs while the tensor pipe
// works for the other.  Each group writes its normalised O rows from registers to global memory and goes on to the
// next item, whose first S tiles the issuer computes meanwhile.
#include "nva_ptx.cuh"
#include "nva_kernels.h"

namespace nva {

namespace {

constexpr int kThreads = 384;           // 4 service warps + 2 softmax warpgroups
constexpr int kSlab = 128 * 128;       // 128 rows x 128 bytes
constexpr int kTile = 2 * kSlab;       // 128 rows x 256 bytes (all 128 dims, or 128 keys of P)
constexpr int kItemRing = 8;           // item descriptors: the producer is at most ~3 items ahead of the softmax warps
constexpr float kNegInf = -__builtin_huge_valf();
constexpr uint32_t kFull = 0xffffffffu;
constexpr float kRescaleLog2 = 8.0f;   // rescale O only when a row maximum grows by more than this (log2 units)

// shared memory map (offsets from a 1024-aligned base)
constexpr int kKStages = 2;
constexpr int kVStages = 3;
constexpr int kOffQ = 0;                              // Q tile of group 0, Q tile of group 1
constexpr int kOffK = kOffQ + 2 * kTile;              // K ring
constexpr int kOffV = kOffK + kKStages * kTile;       // V ring
constexpr int kOffBars = kOffV + kVStages * kTile;    // 40 x u64
constexpr int kOffItems = kOffBars + 40 * 8;          // kItemRing x 2 x int4
constexpr int kOffTmem = kOffItems + kItemRing * 32;
constexpr int kOffAbort = kOffTmem + 4;
constexpr int kSmemBytes = kOffAbort + 4;             // the dynamic shared memory base is 1024-aligned (checked)
static_assert(kSmemBytes <= 232448, "prefill shared memory budget");

// barriers; "w" entries come in pairs, one per query tile of the item (softmax group w)
enum {
  B_QFULL = 0, B_QEMPTY = 2, B_KFULL = 4, B_KEMPTY = 6, B_VFULL = 8, B_VEMPTY = 11, B_SFULL = 14, B_PFULL = 16,
  B_ODONE = 18, B_ITEM = 20,
  B_IREAD = 28   // kItemRing: every consuming warp has read the entry (B_IREAD + kItemRing <= 40)
};
// warps that read each item descriptor: the V producer, the issuer and the eight softmax warps
constexpr int kItemReaders = 10;

struct Item {
  int b, qp, h;        // sequence, query tile pair (tiles 2 qp and 2 qp + 1), q head
  int n, L, q0, k0;    // query rows, keys, first query row, first key row (contiguous K/V only)
  int nkv0, nkv1;      // key tiles under the causal mask of each tile (0: the tile does not exist)
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
  it.qp = e & 0xfff;
  it.h = k - pidx * p.num_heads;
  it.q0 = __ldg(p.cu_q + it.b);
  it.n = __ldg(p.cu_q + it.b + 1) - it.q0;
  it.k0 = __ldg(p.cu_k + it.b);
  it.L = __ldg(p.cu_k + it.b + 1) - it.k0;
  it.nkv0 = prefill_tile_nkv(it.n, it.L, 2 * it.qp);
  it.nkv1 = prefill_tile_nkv(it.n, it.L, 2 * it.qp + 1);
  return it;
}

// ------------------------------------------------------------------------------------------------ main kernel
__global__ void __launch_bounds__(kThreads, 1)
prefill_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if ((smem_u32(smem_raw) & 1023u) != 0) {   // the swizzled layouts need a 1024-byte aligned base
    if (threadIdx.x == 0) atomicOr(&g_error_word, kErrTimeout);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  int4* items = reinterpret_cast<int4*>(smem + kOffItems);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + kOffAbort);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool paged = p.block_tables != nullptr;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_QFULL + i], 1);
      mbar_init(&bars[B_QEMPTY + i], 1);
      mbar_init(&bars[B_KFULL + i], 1);
      mbar_init(&bars[B_KEMPTY + i], 1);
      mbar_init(&bars[B_SFULL + i], 1);
      mbar_init(&bars[B_PFULL + i], 128);
      mbar_init(&bars[B_ODONE + i], 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(&bars[B_VFULL + i], 1);
      mbar_init(&bars[B_VEMPTY + i], 1);
    }
    for (int i = 0; i < kItemRing; ++i) {
      mbar_init(&bars[B_ITEM + i], 1);
      mbar_init(&bars[B_IREAD + i], kItemReaders);
    }
    *abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
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
    int g = 0, qn0 = 0, qn1 = 0;
    bool stop = false;
    int* counter = p.plan + 1 + p.q_tiles_bound;
    // The K producer takes each item and publishes it (nkv = 0: no more items) in the item ring; the V producer,
    // the UMMA issuer and the softmax warps follow the ring, and each of those warps reports on B_IREAD that it has
    // read an entry, which the producer waits for before it writes the entry again (softmax group 1 skips the items
    // without a second tile, so no other wait bounds how far it may lag).
    for (int it_count = 0; !stop; ++it_count) {
      const int e = it_count % kItemRing;
      Item it;
      if (is_k) {
        if (it_count >= kItemRing &&
            !mbar_wait_warp(&bars[B_IREAD + e], ((it_count / kItemRing) + 1) & 1, abort))
          break;
        int k = blockIdx.x;
        if (it_count > 0) {
          int v = 0;
          if (elect_one()) v = atomicAdd(counter, 1);
          k = gridDim.x + __reduce_add_sync(kFull, v);
        }
        it = load_item(p, k, total);   // invalid once k >= number of pairs x heads
        if (elect_one()) {
          items[2 * e] = it.valid ? make_int4(it.b, it.qp, it.h, max(it.nkv0, it.nkv1)) : make_int4(0, 0, 0, 0);
          items[2 * e + 1] = it.valid ? make_int4(it.n, it.L, it.q0, (it.nkv0 << 16) | it.nkv1) : make_int4(0, 0, 0, 0);
          mbar_arrive(&bars[B_ITEM + e]);
        }
        __syncwarp();
        if (!it.valid) break;
      } else {
        if (!mbar_wait_warp(&bars[B_ITEM + e], (it_count / kItemRing) & 1, abort)) break;
        const int4 i0 = items[2 * e];
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_IREAD + e]);
        if (i0.w == 0) break;
        it.b = i0.x;
        it.h = i0.z;
        it.nkv0 = i0.w;   // only the count of key tiles is used below
        it.nkv1 = 0;
        it.k0 = paged ? 0 : __ldg(p.cu_k + it.b);
      }
      const int nkv = max(it.nkv0, it.nkv1);
      const int kvh = it.h / p.group;
      if (is_k) {
        for (int w = 0; w < 2; ++w) {
          if ((w == 0 ? it.nkv0 : it.nkv1) == 0) continue;
          const int qn = w == 0 ? qn0++ : qn1++;
          if (!mbar_wait_warp(&bars[B_QEMPTY + w], (qn & 1) ^ 1, abort)) {
            stop = true;
            break;
          }
          if (elect_one()) {
            mbar_arrive_expect_tx(&bars[B_QFULL + w], kTile);
            uint8_t* dst = smem + kOffQ + w * kTile;
            const int row = it.q0 + (2 * it.qp + w) * 128;
            tma_load_3d(dst, &tm_q, 0, it.h, row, &bars[B_QFULL + w]);
            tma_load_3d(dst + kSlab, &tm_q, 64, it.h, row, &bars[B_QFULL + w]);
          }
          __syncwarp();
        }
      }
      for (int base = 0; base < nkv && !stop; base += 32) {
        // key-tile rows for the next 32 tiles (block-table reads in parallel across lanes)
        int row0 = 0;
        if (base + lane < nkv) {
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
        const int cnt = min(32, nkv - base);
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
    // Per item, with n0 / n1 key tiles for the two query tiles (n1 = 0 or n0 <= n1 <= n0 + 1):
    //   S0(0), S1(0), then for each key tile j: PV0(j), S0(j+1), PV1(j), S1(j+1)
    // (products that do not exist are skipped).  S_w(j+1) overwrites the TMEM columns that hold P_w(j), so it
    // follows PV_w(j) (the tensor pipe runs one thread's products in issue order); in the same way the commit that
    // reports S_w(j) also covers PV_w(j-1), so a softmax group that sees S_w(j) may rescale O_w.
    constexpr uint32_t idesc_qk = umma_idesc_bf16(128, 128, false, false);
    constexpr uint32_t idesc_pv = umma_idesc_bf16(128, 128, false, true);
    const uint64_t q_desc0 = umma_desc_sw128(smem_u32(smem + kOffQ), 16, 1024);
    const uint64_t k_desc0 = umma_desc_sw128(smem_u32(smem + kOffK), 16, 1024);
    const uint64_t v_desc0 = umma_desc_sw128(smem_u32(smem + kOffV), kSlab, 1024);
    int gk = 0, gv = 0, gq0 = 0, gq1 = 0, gpv0 = 0, gpv1 = 0;
    bool ok = true;
    for (int it_count = 0; ok; ++it_count) {
      const int e = it_count % kItemRing;
      if (!mbar_wait_warp(&bars[B_ITEM + e], (it_count / kItemRing) & 1, abort)) break;
      const int4 i0 = items[2 * e], i1 = items[2 * e + 1];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_IREAD + e]);
      const int nkv = i0.w;
      if (nkv == 0) break;
      const int n0 = i1.w >> 16, n1 = i1.w & 0xffff;
      int k_seen = -1, v_seen = -1;
      auto qk = [&](int w, int j) {
        if (!ok) return;
        if (j == 0) {
          const int qn = w == 0 ? gq0 : gq1;
          if (!mbar_wait_warp(&bars[B_QFULL + w], qn & 1, abort)) { ok = false; return; }
        }
        const int kt = gk + j, st = kt % kKStages;
        if (j > k_seen) {
          if (!mbar_wait_warp(&bars[B_KFULL + st], (kt / kKStages) & 1, abort)) { ok = false; return; }
          k_seen = j;
        }
        tc_fence_after();
        if (elect_one()) {
          // K-major SW128 operands: step k sits at +32 B within a 128-byte row, steps 4..7 in the second slab
          constexpr uint32_t kOff[8] = {0, 2, 4, 6, kSlab >> 4, (kSlab >> 4) + 2, (kSlab >> 4) + 4, (kSlab >> 4) + 6};
          umma_bf16_ss_x8(tmem + w * 128, q_desc0 + ((w * kTile) >> 4), k_desc0 + ((st * kTile) >> 4), idesc_qk, 0u,
                          kOff, kOff);
          umma_commit(&bars[B_SFULL + w]);
          if (w == 1 || j >= n1) umma_commit(&bars[B_KEMPTY + st]);       // last reader of this K tile
          if (j == (w == 0 ? n0 : n1) - 1) umma_commit(&bars[B_QEMPTY + w]);
        }
        __syncwarp();
      };
      auto pv = [&](int w, int j) {
        if (!ok) return;
        int& gp = w == 0 ? gpv0 : gpv1;
        if (!mbar_wait_warp(&bars[B_PFULL + w], gp & 1, abort)) { ok = false; return; }
        const int vt = gv + j, st = vt % kVStages;
        if (j > v_seen) {
          if (!mbar_wait_warp(&bars[B_VFULL + st], (vt / kVStages) & 1, abort)) { ok = false; return; }
          v_seen = j;
        }
        tc_fence_after();
        if (elect_one()) {
          const uint64_t vd = v_desc0 + ((st * kTile) >> 4);
          const uint32_t pa = tmem + w * 128;   // P_w(j): first 64 columns of S_w
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)   // V: 16 keys (2048 B) per step; P: 8 columns per step; fresh O per item
            umma_bf16_ts(tmem + 256 + w * 128, pa + kk * 8, vd + kk * (2048 >> 4), idesc_pv,
                         (j > 0 || kk > 0) ? 1u : 0u);
          if (w == 1 || j >= n1) umma_commit(&bars[B_VEMPTY + st]);       // last reader of this V tile
          if (j == (w == 0 ? n0 : n1) - 1) umma_commit(&bars[B_ODONE + w]);
        }
        __syncwarp();
        ++gp;
      };
      if (n0 > 0) qk(0, 0);
      if (n1 > 0) qk(1, 0);
      for (int j = 0; j < nkv && ok; ++j) {
        if (j < n0) {
          pv(0, j);
          if (j + 1 < n0) qk(0, j + 1);
        }
        if (j < n1) {
          pv(1, j);
          if (j + 1 < n1) qk(1, j + 1);
        }
      }
      gk += nkv;
      gv += nkv;
      if (n0 > 0) ++gq0;
      if (n1 > 0) ++gq1;
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue: one warpgroup per query tile
    const int w = (warp - 4) >> 2;            // query tile of the item
    const int wq = warp & 3;                  // TMEM lane quadrant
    const int t = wq * 32 + lane;             // query row within the tile
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    const uint32_t s_col = w * 128, o_col = 256 + w * 128;
    int gs = 0, go = 0, gvv = 0;              // S tiles seen, items finished, V tiles of earlier items
    bool alive = true;
    for (int it_count = 0; alive; ++it_count) {
      const int e = it_count % kItemRing;
      if (!mbar_wait_warp(&bars[B_ITEM + e], (it_count / kItemRing) & 1, abort)) break;
      const int4 i0 = items[2 * e], i1 = items[2 * e + 1];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_IREAD + e]);
      const int nkv = i0.w;
      if (nkv == 0) break;
      const int n0 = i1.w >> 16, n1 = i1.w & 0xffff;
      const int nw = w == 0 ? n0 : n1;
      const int vbase = gvv;
      gvv += nkv;
      if (nw == 0) continue;
      const int n = i1.x, L = i1.y, qt = 2 * i0.y + w;
      const int rows = min(128, n - qt * 128);
      const int lim = L - n + qt * 128 + t;   // this row sees keys <= lim
      float m_used = kNegInf, l = 0.f;
      for (int j = 0; j < nw && alive; ++j, ++gs) {
        // paged keys past the sequence end may be stale or uninitialised: zero V there (P is 0 there anyway).
        // The first group that reads the tile (group 0 unless the tile is group 1's alone) does it before its P.
        if (paged && j * 128 + 127 >= L && w == (j < n0 ? 0 : 1)) {
          const int vt = vbase + j, vs = vt % kVStages;
          alive = mbar_wait_warp(&bars[B_VFULL + vs], (vt / kVStages) & 1, abort);
          if (alive && j * 128 + t >= L) {
            uint8_t* vrow = smem + kOffV + vs * kTile + t * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0u, 0u, 0u, 0u);
              *reinterpret_cast<uint4*>(vrow + kSlab + c * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
            // generic-proxy writes, read by the PV product through the async proxy: ordered by this fence and
            // this thread's later PFULL arrival
            fence_proxy_async_smem();
          }
          if (!alive) break;
        }
        alive = mbar_wait_warp(&bars[B_SFULL + w], gs & 1, abort);
        if (!alive) break;
        tc_fence_after();
        // Online softmax in two 64-key halves: each half loads its S columns once, updates the row maximum and
        // writes its P (keys [64 h, 64 h + 64) -> columns [32 h, 32 h + 32) of S_w, which the first half has
        // already read).  When the second half raises the maximum past the rescale threshold, O, l and the first
        // half's P are scaled down to the new maximum.
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float s[64];
          tmem_ld64(t_lane + s_col + 64 * h, s);
          const int kmax = lim - j * 128 - 64 * h;     // columns > kmax of this half are masked for this row
          if (kmax < 63) {
#pragma unroll
            for (int c = 0; c < 64; ++c) s[c] = c <= kmax ? s[c] : kNegInf;
          }
          // Weights against the running maximum.  A half-row sum below 2^8 shows that no weight reached 2^8, i.e.
          // this half did not raise the maximum past the rescale threshold: the half is done without computing its
          // maximum.  Otherwise (or before the row's first key) the warp takes the exact path: maximum, rescale,
          // weights again.  Masked keys hold -inf, so their weights are exp2(-inf) = 0; a row that has seen no key
          // yet (m_used = -inf) subtracts 0 and gets only zeros.
          float pk[32];
          float hsum = 0.f;
          auto weights = [&]() {
            const float neg_m = m_used == kNegInf ? 0.f : -m_used;
            const float2 nm2 = make_float2(neg_m, neg_m);
            float2 sum4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                              make_float2(0.f, 0.f)};
#pragma unroll
            for (int c = 0; c < 64; c += 2) {
              const float2 x = ffma2(make_float2(s[c], s[c + 1]), sc2, nm2);
              const float2 pp = make_float2(fast_exp2(x.x), fast_exp2(x.y));
              sum4[(c >> 1) & 3] = fadd2(sum4[(c >> 1) & 3], pp);
              pk[c >> 1] = __uint_as_float(pack_bf16x2(pp.x, pp.y));
            }
            const float2 s01 = fadd2(fadd2(sum4[0], sum4[1]), fadd2(sum4[2], sum4[3]));
            hsum = s01.x + s01.y;
          };
          bool exact = m_used == kNegInf;
          if (!__any_sync(kFull, exact)) {
            weights();
            exact = !(hsum < 256.f);
          }
          if (__any_sync(kFull, exact)) {
            float m8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              m8[i] = fmaxf(fmax3(fmax3(s[i], s[i + 8], s[i + 16]), s[i + 24], s[i + 32]),
                            fmax3(s[i + 40], s[i + 48], s[i + 56]));
            const float mx = fmaxf(fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), m8[6]), m8[7]);
            const float m_cand = fmaxf(m_used, mx * p.scale_log2);
            const bool rescale = m_used != kNegInf && m_cand > m_used + kRescaleLog2;
            if (__any_sync(kFull, rescale)) {
              const float alpha = rescale ? fast_exp2(m_used - m_cand) : 1.f;
              if (j > 0) {
                // the commit that reported S_w(j) also covers PV_w(j-1): O_w holds every earlier product of the item
#pragma unroll 1
                for (int c = 0; c < 128; c += 32) {
                  float ot[32];
                  tmem_ld32(t_lane + o_col + c, ot);
#pragma unroll
                  for (int i = 0; i < 32; ++i) ot[i] *= alpha;
                  tmem_st32(t_lane + o_col + c, ot);
                }
              }
              if (h == 1) {   // the first half's P was taken against the old maximum
                tmem_wait_st();
                float pv[32];
                tmem_ld32(t_lane + s_col, pv);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                  const uint32_t u = __float_as_uint(pv[i]);
                  pv[i] = __uint_as_float(pack_bf16x2(__uint_as_float(u << 16) * alpha,
                                                      __uint_as_float(u & 0xffff0000u) * alpha));
                }
                tmem_st32(t_lane + s_col, pv);
              }
              if (rescale) l *= alpha;
            }
            if (rescale || m_used == kNegInf) m_used = m_cand;
            weights();
          }
          tmem_st32_nowait(t_lane + s_col + 32 * h, pk);
          l += hsum;
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&bars[B_PFULL + w]);
      }
      if (!alive) break;
      // ---- epilogue: O_w / l straight from TMEM to the output rows (one 256-byte row per thread)
      alive = mbar_wait_warp(&bars[B_ODONE + w], go & 1, abort);
      ++go;
      if (!alive) break;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.out + (int64_t)(i1.z + qt * 128 + t) * p.out_row_stride + (int64_t)i0.z * kHeadDim;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        float ot[32];
        tmem_ld32(t_lane + o_col + c, ot);
        if (t < rows) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            v.x = pack_bf16x2(ot[i] * inv, ot[i + 1] * inv);
            v.y = pack_bf16x2(ot[i + 2] * inv, ot[i + 3] * inv);
            v.z = pack_bf16x2(ot[i + 4] * inv, ot[i + 5] * inv);
            v.w = pack_bf16x2(ot[i + 6] * inv, ot[i + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c + i) = v;
          }
        }
      }
      // O_w is read: the next item's PV_w(0), which overwrites it, follows this thread's next PFULL arrival
      tc_fence_before();
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

cudaError_t launch_prefill_pair(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                                const PrefillParams& p, int grid, cudaStream_t stream) {
  if (p.num_seqs > kMaxDecodeSeqs || p.q_tiles_bound > kMaxPrefillTiles || p.tiles_per_item != 2)
    return cudaErrorInvalidValue;
  const cudaError_t e =
      cudaFuncSetAttribute(prefill_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  return launch_kernel(prefill_pair_kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, true, tm_q, tm_k, tm_v, p);
}

}  // namespace nva
