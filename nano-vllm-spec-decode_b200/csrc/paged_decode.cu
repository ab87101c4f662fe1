// Paged GQA decode / speculative-verify attention for sm_100a (replaces flash_attn_with_kvcache at
// nanovllm/layers/attention.py:75-77 and the short-query rows of flash_attn_varlen_func in mixed batches).
//
// Orientation ("swap AB"): the 128 tokens of a KV tile sit on the 128 TMEM lanes (UMMA M) and the query rows of
// one kv head -- q_len draft positions x group q heads, packed row r = i * group + h -- sit on UMMA N (16/32/48).
//   S^T[tok, r] = K[tok, :] . Q[r, :]        (A = K tile, K-major;  B = Q rows, K-major)
//   O^T[d, r]   = sum_tok V[tok, d] P[tok, r] (A = V tile, MN-major; B = P^T, K-major)
// so one HBM pass over each KV block serves every q head of its group and every draft position.
//
// Work split: every CTA is persistent (one per SM) and owns an equal share of the 128-token tiles of all
// (sequence, kv head) segments, in (sequence, kv head, tile) order.  A segment that lies inside one CTA is
// finished there; one cut by a CTA boundary leaves a normalised partial + log2-sum-exp per piece, merged by
// paged_decode_combine.  The split depends only on the batch's lengths, so padding sequences (length 0) change
// nothing, and no host value or device read-back is involved (graph-capturable, fixed launch geometry).
//
// Warp roles (256 threads): 0 = TMA producer (K and V tiles, 4 boxes of 64 dims x 128 tokens per stage),
// 1 = TMEM owner + single-thread UMMA issuer, 2 = Q loader (gathers a segment's rows into the 128B-swizzled
// operand layout), 3 = idle, 4..7 = softmax / accumulation (thread ct owns TMEM lane ct: token ct of S^T and
// dim ct of O^T).
#include "nva_ptx.cuh"
#include "nva_kernels.h"

namespace nva {

namespace {

constexpr int kStages = 3;
constexpr int kSlab = 128 * 128;            // 128 rows x 128 bytes
constexpr int kStageBytes = 4 * kSlab;      // K lo, K hi, V lo, V hi
constexpr int kThreads = 256;
constexpr int kConsumerBase = 128;          // first softmax thread
constexpr float kNegInf = -__builtin_huge_valf();

template <int NP>
struct Smem {
  static constexpr int kQ = kStages * kStageBytes;
  static constexpr int kP = kQ + NP * 256;
  static constexpr int kMisc = kP + NP * 256;
  // misc block
  static constexpr int kBars = kMisc;                         // 16 x u64
  static constexpr int kInfo = kBars + 16 * 8;                // kStages x int4
  static constexpr int kRed = kInfo + kStages * 16;           // [2][4][NP] float
  static constexpr int kM = kRed + 2 * 4 * NP * 4;            // [NP]
  static constexpr int kAlpha = kM + NP * 4;                  // [2][NP]
  static constexpr int kLred = kAlpha + 2 * NP * 4;           // [4][NP]
  static constexpr int kTmem = kLred + 4 * NP * 4;            // u32
  static constexpr int kAbort = kTmem + 4;                    // int
  static constexpr int kScan = kAbort + 4;                    // [8] int (warp totals)
  static constexpr int kPrefix = kScan + 8 * 4;               // [kMaxDecodeSeqs + 1] int
  static constexpr int kEnd = kPrefix + (kMaxDecodeSeqs + 1) * 4;
  static constexpr int kBytes = kEnd + 1024;                  // + slack for 1024-byte alignment
};

// barrier indices
enum { B_KV_FULL = 0, B_KV_EMPTY = 3, B_S_FULL = 6, B_S_EMPTY = 8, B_P_FULL = 10, B_O_FULL = 11, B_Q_FULL = 12,
       B_Q_EMPTY = 13 };

struct SeqShape {
  int n;   // query rows
  int L;   // keys
  int q0;  // first query row
};

__device__ __forceinline__ SeqShape seq_shape(const DecodeParams& p, int b) {
  SeqShape s;
  if (p.cu_q != nullptr) {
    const int a = __ldg(p.cu_q + b);
    s.n = __ldg(p.cu_q + b + 1) - a;
    s.q0 = a;
    s.L = __ldg(p.cu_k + b + 1) - __ldg(p.cu_k + b);
  } else {
    s.n = p.n_fixed;
    s.q0 = b * p.n_fixed;
    s.L = __ldg(p.ctx_lens + b);
  }
  return s;
}

__device__ __forceinline__ int seq_tiles(const DecodeParams& p, int b) {
  const SeqShape s = seq_shape(p, b);
  if (s.n < 1 || s.n > p.max_n || s.L < 1) return 0;
  return (s.L + kTileTokens - 1) / kTileTokens;
}

// Exclusive prefix sum of per-sequence tile counts into prefix[0..B] (prefix[B] = total per kv head).
// Called by all `nthreads` threads of the block; ends with a __syncthreads.
__device__ void build_prefix(const DecodeParams& p, int* prefix, int* warp_tot, int tid, int nthreads) {
  const int lane = tid & 31, warp = tid >> 5, nwarps = nthreads >> 5;
  int running = 0;
  for (int base = 0; base < p.num_seqs; base += nthreads) {
    const int b = base + tid;
    const int v = b < p.num_seqs ? seq_tiles(p, b) : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    int before = running;
    int chunk = 0;
    for (int w = 0; w < nwarps; ++w) {
      if (w < warp) before += warp_tot[w];
      chunk += warp_tot[w];
    }
    if (b < p.num_seqs) prefix[b] = before + x - v;
    running += chunk;
    __syncthreads();
  }
  if (tid == 0) prefix[p.num_seqs] = running;
  __syncthreads();
}

struct Loc {
  int b, g, j, nt, s0;
};

// Global tile t -> (sequence, kv head, tile within segment).  Requires t < KVH * prefix[B].
__device__ __forceinline__ Loc locate(int t, const int* prefix, int B, int KVH) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (KVH * prefix[mid] <= t) lo = mid; else hi = mid - 1;
  }
  Loc l;
  l.b = lo;
  l.nt = prefix[lo + 1] - prefix[lo];
  const int rem = t - KVH * prefix[lo];
  l.g = rem / l.nt;
  l.j = rem - l.g * l.nt;
  l.s0 = KVH * prefix[lo] + l.g * l.nt;
  return l;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int NP>
__global__ void __launch_bounds__(kThreads, 1)
paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                    const DecodeParams p) {
  using L = Smem<NP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
  int4* info = reinterpret_cast<int4*>(smem + L::kInfo);
  float* red = reinterpret_cast<float*>(smem + L::kRed);
  float* m_s = reinterpret_cast<float*>(smem + L::kM);
  float* alpha_s = reinterpret_cast<float*>(smem + L::kAlpha);
  float* lred = reinterpret_cast<float*>(smem + L::kLred);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + L::kAbort);
  int* warp_tot = reinterpret_cast<int*>(smem + L::kScan);
  int* prefix = reinterpret_cast<int*>(smem + L::kPrefix);
  uint8_t* q_smem = smem + L::kQ;
  uint8_t* p_smem = smem + L::kP;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int KVH = p.num_kv_heads;
  const int G = p.group;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[B_KV_FULL + s], 1);
      mbar_init(&bars[B_KV_EMPTY + s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_S_FULL + i], 1);
      mbar_init(&bars[B_S_EMPTY + i], 128);
    }
    mbar_init(&bars[B_P_FULL], 128);
    mbar_init(&bars[B_O_FULL], 1);
    mbar_init(&bars[B_Q_FULL], 32);
    mbar_init(&bars[B_Q_EMPTY], 1);
    *abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  build_prefix(p, prefix, warp_tot, tid, kThreads);   // ends with __syncthreads
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int total = KVH * prefix[p.num_seqs];
  const int per = total > 0 ? (total + gridDim.x - 1) / gridDim.x : 1;
  const int t_begin = blockIdx.x * per;
  const int t_end = min(total, t_begin + per);
  const int ntiles = t_end > t_begin ? t_end - t_begin : 0;

  if (warp == 0 && ntiles > 0) {
    // ------------------------------------------------------------ TMA producer (whole warp waits, lane 0 issues)
    for (int jj = 0; jj < ntiles; ++jj) {
      const int t = t_begin + jj;
      const int stage = jj % kStages;
      if (!mbar_wait_warp(&bars[B_KV_EMPTY + stage], ((jj / kStages) & 1) ^ 1, abort)) break;
      if (lane == 0) {
        const Loc lc = locate(t, prefix, p.num_seqs, KVH);
        const int tok0 = lc.j * kTileTokens;
        int page = __ldg(p.block_tables + (int64_t)lc.b * p.bt_stride + tok0 / p.block_size);
        if (page < 0 || page >= p.num_blocks) {
          atomicOr(&g_error_word, kErrBlockRange);
          page = -1;   // TMA fills out-of-range rows with zeros; nothing outside the pool is read
        }
        const int row0 = page * p.block_size + (tok0 % p.block_size);
        const int flags = (lc.j == 0 || t == t_begin ? 1 : 0) | (lc.j == lc.nt - 1 || t == t_end - 1 ? 2 : 0);
        info[stage] = make_int4(lc.b, lc.g, lc.j, flags);
        uint64_t* full = &bars[B_KV_FULL + stage];
        mbar_arrive_expect_tx(full, kStageBytes);
        uint8_t* dst = smem + stage * kStageBytes;
        tma_load_3d(dst, &tm_k, 0, lc.g, row0, full);
        tma_load_3d(dst + kSlab, &tm_k, 64, lc.g, row0, full);
        tma_load_3d(dst + 2 * kSlab, &tm_v, 0, lc.g, row0, full);
        tma_load_3d(dst + 3 * kSlab, &tm_v, 64, lc.g, row0, full);
      }
      __syncwarp();
    }
  } else if (warp == 1 && ntiles > 0) {
    // ------------------------------------------------------------ UMMA issuer (whole warp waits, lane 0 issues)
    constexpr uint32_t idesc_qk = umma_idesc_bf16(128, NP, false, false);
    constexpr uint32_t idesc_pv = umma_idesc_bf16(128, NP, true, false);
    const uint32_t q_base = smem_u32(q_smem);
    const uint32_t p_base = smem_u32(p_smem);
    const uint32_t kv_base = smem_u32(smem);
    int qi = 0;
    auto issue_pv = [&](int ii) -> bool {
      const int st = ii % kStages;
      if (!mbar_wait_warp(&bars[B_P_FULL], ii & 1, abort)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t v_lo = kv_base + st * kStageBytes + 2 * kSlab;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t a = umma_desc_sw128(v_lo + k * 2048, kSlab, 1024);
          const uint64_t b = umma_desc_sw128(p_base + (k >> 2) * (NP * 128) + (k & 3) * 32, 16, 1024);
          umma_bf16_ss(tmem + 2 * NP, a, b, idesc_pv, k > 0);
        }
        umma_commit(&bars[B_O_FULL]);
        umma_commit(&bars[B_KV_EMPTY + st]);
      }
      __syncwarp();
      return true;
    };
    bool ok = true;
    for (int jj = 0; jj < ntiles && ok; ++jj) {
      const int st = jj % kStages;
      if (!mbar_wait_warp(&bars[B_KV_FULL + st], (jj / kStages) & 1, abort)) { ok = false; break; }
      const int4 inf = info[st];
      if (inf.w & 1) {
        if (!mbar_wait_warp(&bars[B_Q_FULL], qi & 1, abort)) { ok = false; break; }
      }
      const int buf = jj & 1;
      if (!mbar_wait_warp(&bars[B_S_EMPTY + buf], ((jj >> 1) & 1) ^ 1, abort)) { ok = false; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t k_lo = kv_base + st * kStageBytes;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t a = umma_desc_sw128(k_lo + (k >> 2) * kSlab + (k & 3) * 32, 16, 1024);
          const uint64_t b = umma_desc_sw128(q_base + (k >> 2) * (NP * 128) + (k & 3) * 32, 16, 1024);
          umma_bf16_ss(tmem + buf * NP, a, b, idesc_qk, k > 0);
        }
        umma_commit(&bars[B_S_FULL + buf]);
        if (inf.w & 2) umma_commit(&bars[B_Q_EMPTY]);
      }
      __syncwarp();
      if (inf.w & 2) ++qi;
      if (jj > 0) ok = issue_pv(jj - 1);
    }
    if (ok) issue_pv(ntiles - 1);
  } else if (warp == 2 && ntiles > 0) {
    // ------------------------------------------------------------ Q loader
    int qi = 0;
    int t = t_begin;
    while (t < t_end) {
      const Loc lc = locate(t, prefix, p.num_seqs, KVH);
      if (!mbar_wait_warp(&bars[B_Q_EMPTY], (qi & 1) ^ 1, abort)) break;
      const SeqShape ss = seq_shape(p, lc.b);
      const int R = ss.n * G;
      for (int idx = lane; idx < NP * 16; idx += 32) {
        const int r = idx >> 4, c = idx & 15;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < R) {
          const int i = r / G, h = r - i * G;
          const __nv_bfloat16* src = p.q + (int64_t)(ss.q0 + i) * p.q_row_stride + (int64_t)(lc.g * G + h) * kHeadDim + c * 8;
          v = __ldg(reinterpret_cast<const uint4*>(src));
        }
        *reinterpret_cast<uint4*>(q_smem + (c >> 3) * (NP * 128) + sw128_offset(r, c & 7)) = v;
      }
      fence_proxy_async_smem();
      __syncwarp();
      mbar_arrive(&bars[B_Q_FULL]);
      ++qi;
      t = lc.s0 + lc.nt;   // next segment
    }
  } else if (warp >= 4 && ntiles > 0) {
    // ------------------------------------------------------------ softmax / accumulation
    // Every wait here is warp-uniform and every named barrier ORs "gave up" across the four warps, so the
    // warps leave the loop together if a wait expires (no warp can be left behind at a barrier).
    const int ct = tid - kConsumerBase;       // TMEM lane: token ct of S^T, dim ct of O^T
    const int wq = ct >> 5;                   // lane quadrant
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    float l[NP], o[NP], s[NP];
    SeqShape ss{0, 0, 0};
    int R = 0, seg_s0 = 0, seg_s1 = 0, seg_g = 0;
    bool alive = true;
    for (int jj = 0; jj < ntiles; ++jj) {
      const int st = jj % kStages;
      const int buf = jj & 1;
      const int rb = jj & 1;
      alive = alive && mbar_wait_warp(&bars[B_KV_FULL + st], (jj / kStages) & 1, abort);
      int4 inf = make_int4(0, 0, 0, 0);
      if (alive) inf = info[st];
      const bool first = inf.w & 1, last = inf.w & 2;
      if (alive && first) {
        seg_g = inf.y;
        ss = seq_shape(p, inf.x);
        R = ss.n * G;
        const int nt = (ss.L + kTileTokens - 1) / kTileTokens;
        seg_s0 = KVH * prefix[inf.x] + seg_g * nt;
        seg_s1 = seg_s0 + nt;
#pragma unroll
        for (int r = 0; r < NP; ++r) { l[r] = 0.f; o[r] = 0.f; }
      }
      const int tok0 = inf.z * kTileTokens;
      const int tok = tok0 + ct;
      // rows past the sequence end may hold stale or uninitialised values: zero V there so P = 0 cannot
      // meet a NaN in the PV product
      if (alive && ss.L - tok0 < kTileTokens && tok >= ss.L) {
        uint8_t* vrow = smem + st * kStageBytes + 2 * kSlab + ct * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(vrow + kSlab + c * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      // ---- S tile -> masked, scaled scores; per-warp column maxima
      alive = alive && mbar_wait_warp(&bars[B_S_FULL + buf], (jj >> 1) & 1, abort);
      if (alive) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < NP; c += 16) tmem_ld16(t_lane + buf * NP + c, s + c);
        tc_fence_before();
        mbar_arrive(&bars[B_S_EMPTY + buf]);
        const int lim = ss.L - ss.n;   // query i sees tokens <= lim + i
#pragma unroll
        for (int r = 0; r < NP; ++r) {
          const bool vis = r < R && tok <= lim + r / G;
          s[r] = vis ? s[r] * p.scale_log2 : kNegInf;
          if (r < R) {
            const float mx = warp_max(s[r]);
            if (lane == 0) red[(rb * 4 + wq) * NP + r] = mx;
          }
        }
      }
      if (named_bar_any(1, 128, !alive)) break;
      // ---- running max (owner thread per row) and rescale factor
      if (ct < R) {
        const float* rr = red + rb * 4 * NP;
        const float tm = fmaxf(fmaxf(rr[ct], rr[NP + ct]), fmaxf(rr[2 * NP + ct], rr[3 * NP + ct]));
        const float mo = first ? kNegInf : m_s[ct];
        const float mn = fmaxf(mo, tm);
        m_s[ct] = mn;
        alpha_s[rb * NP + ct] = (mn == kNegInf) ? 1.f : fast_exp2(mo - mn);
      }
      named_bar_sync(1, 128);
#pragma unroll
      for (int r = 0; r < NP; ++r) {
        if (r < R) {
          const float pr = (s[r] == kNegInf) ? 0.f : fast_exp2(s[r] - m_s[r]);
          l[r] = l[r] * alpha_s[rb * NP + r] + pr;
          s[r] = pr;
        } else {
          s[r] = 0.f;
        }
      }
      // ---- fold the previous tile's O; PV of tile jj-1 must be done before P is overwritten
      if (!first) {
        alive = mbar_wait_warp(&bars[B_O_FULL], (jj - 1) & 1, abort);
        if (alive) {
          tc_fence_after();
          float ot[16];
#pragma unroll
          for (int c = 0; c < NP; c += 16) {
            tmem_ld16(t_lane + 2 * NP + c, ot);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[c + i] = o[c + i] * alpha_s[(rb ^ 1) * NP + c + i] + ot[i];
          }
          tc_fence_before();
        }
      }
      // ---- P^T (bf16) into the K-major 128B-swizzled B operand: row r, token ct
      if (alive) {
        uint8_t* pb = p_smem + (ct >> 6) * (NP * 128);
        const uint32_t chunk = (ct & 63) >> 3, sub = (ct & 7) * 2;
#pragma unroll
        for (int r = 0; r < NP; ++r)
          *reinterpret_cast<__nv_bfloat16*>(pb + sw128_offset(r, chunk) + sub) = __float2bfloat16_rn(s[r]);
        fence_proxy_async_smem();
        mbar_arrive(&bars[B_P_FULL]);
      }
      if (last && alive) {
        alive = mbar_wait_warp(&bars[B_O_FULL], jj & 1, abort);
        if (alive) {
          tc_fence_after();
          float ot[16];
#pragma unroll
          for (int c = 0; c < NP; c += 16) {
            tmem_ld16(t_lane + 2 * NP + c, ot);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[c + i] = o[c + i] * alpha_s[rb * NP + c + i] + ot[i];
          }
          tc_fence_before();
#pragma unroll
          for (int r = 0; r < NP; ++r) {
            if (r < R) {
              const float sm = warp_sum(l[r]);
              if (lane == 0) lred[wq * NP + r] = sm;
            }
          }
        }
      }
      if (named_bar_any(1, 128, !alive)) break;
      if (last) {
        const bool complete = (seg_s0 / per) == ((seg_s1 - 1) / per);
        const int slot = 2 * blockIdx.x + (seg_s0 < t_begin ? 0 : 1);
#pragma unroll
        for (int r = 0; r < NP; ++r) {
          if (r < R) {
            const float lt = lred[r] + lred[NP + r] + lred[2 * NP + r] + lred[3 * NP + r];
            const float val = lt > 0.f ? o[r] / lt : 0.f;
            if (complete) {
              const int i = r / G, h = r - i * G;
              p.out[(int64_t)(ss.q0 + i) * p.out_row_stride + (int64_t)(seg_g * G + h) * kHeadDim + ct] =
                  __float2bfloat16_rn(val);
            } else {
              p.part_o[((int64_t)slot * NP + r) * kHeadDim + ct] = val;
              if (ct == 0) p.part_lse[slot * NP + r] = lt > 0.f ? m_s[r] + __log2f(lt) : kNegInf;
            }
          }
        }
      }
    }
  }

  __syncthreads();
  if (*abort) {
    // a wait gave up: let any copy or MMA still in flight land before the shared memory and TMEM go away
    if (tid == 0) atomicOr(&g_error_word, kErrTimeout);
    for (int i = 0; i < 1000; ++i) sleep_ns(1000);
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// Merge the pieces of segments cut by CTA boundaries, and zero the rows of sequences with no keys.
template <int NP>
__global__ void __launch_bounds__(128)
paged_decode_combine(const DecodeParams p, int main_grid) {
  __shared__ int prefix[kMaxDecodeSeqs + 1];
  __shared__ int warp_tot[4];
  const int tid = threadIdx.x;
  build_prefix(p, prefix, warp_tot, tid, 128);
  const int KVH = p.num_kv_heads, G = p.group;
  // zero-length sequences (batch padding): their rows see no key, output 0
  for (int b = blockIdx.x; b < p.num_seqs; b += gridDim.x) {
    const SeqShape ss = seq_shape(p, b);
    if (ss.n >= 1 && ss.n <= p.max_n && ss.L < 1) {
      for (int i = 0; i < ss.n; ++i)
        for (int h = 0; h < p.num_heads; ++h)
          p.out[(int64_t)(ss.q0 + i) * p.out_row_stride + (int64_t)h * kHeadDim + tid] = __float2bfloat16_rn(0.f);
    }
  }
  const int total = KVH * prefix[p.num_seqs];
  const int per = total > 0 ? (total + main_grid - 1) / main_grid : 1;
  for (int c = blockIdx.x; c < main_grid; c += gridDim.x) {
    const int t = c * per;
    if (c == 0 || t >= total) continue;
    const Loc lc = locate(t, prefix, p.num_seqs, KVH);
    const int s1 = lc.s0 + lc.nt;
    if (lc.s0 >= t || (s1 - 1) / per != c) continue;   // not a cut segment ending in CTA c
    const int c0 = lc.s0 / per;
    const SeqShape ss = seq_shape(p, lc.b);
    const int R = ss.n * G;
    for (int r = 0; r < R; ++r) {
      float mx = p.part_lse[(2 * c0 + 1) * NP + r];
      for (int cc = c0 + 1; cc <= c; ++cc) mx = fmaxf(mx, p.part_lse[(2 * cc) * NP + r]);
      float acc = 0.f, den = 0.f;
      if (mx != kNegInf) {
        for (int cc = c0; cc <= c; ++cc) {
          const int slot = cc == c0 ? 2 * c0 + 1 : 2 * cc;
          const float lse = p.part_lse[slot * NP + r];
          const float w = lse == kNegInf ? 0.f : fast_exp2(lse - mx);
          acc += w * p.part_o[((int64_t)slot * NP + r) * kHeadDim + tid];
          den += w;
        }
      }
      const int i = r / G, h = r - i * G;
      p.out[(int64_t)(ss.q0 + i) * p.out_row_stride + (int64_t)(lc.g * G + h) * kHeadDim + tid] =
          __float2bfloat16_rn(den > 0.f ? acc / den : 0.f);
    }
  }
}

template <int NP>
cudaError_t launch_np(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const DecodeParams& p, int grid,
                      cudaStream_t stream) {
  constexpr int smem = Smem<NP>::kBytes;
  static_assert(smem <= 232448, "shared memory budget");
  cudaError_t e = cudaFuncSetAttribute(paged_decode_kernel<NP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  paged_decode_kernel<NP><<<grid, kThreads, smem, stream>>>(tm_k, tm_v, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  paged_decode_combine<NP><<<grid, 128, 0, stream>>>(p, grid);
  return cudaGetLastError();
}

}  // namespace

int decode_rows_padded(int rows) {
  if (rows <= 16) return 16;
  if (rows <= 32) return 32;
  if (rows <= 48) return 48;
  return 0;
}

size_t decode_workspace_bytes(int grid, int np) {
  return static_cast<size_t>(2) * grid * np * (kHeadDim + 1) * sizeof(float) + 256;
}

cudaError_t launch_paged_decode(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const DecodeParams& p, int np,
                                int grid, cudaStream_t stream) {
  switch (np) {
    case 16: return launch_np<16>(tm_k, tm_v, p, grid, stream);
    case 32: return launch_np<32>(tm_k, tm_v, p, grid, stream);
    case 48: return launch_np<48>(tm_k, tm_v, p, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nva
