// Paged GQA decode / speculative-verify attention for sm_100a (replaces flash_attn_with_kvcache at
// nanovllm/layers/attention.py:75-77 and the short-query rows of flash_attn_varlen_func in mixed batches).
//
// Orientation ("swap AB"): the 128 tokens of a KV tile sit on the 128 TMEM lanes (UMMA M) and the query rows of
// one kv head -- q_len draft positions x group q heads, packed row r = i * group + h -- sit on UMMA N (16/32/48):
//   S^T[tok, r] = K[tok, :] . Q[r, :]          A = K tile (K-major, 128B swizzle, straight from TMA)
//                                              B = Q rows (K-major, 128B swizzle, gathered with cp.async)
//   O^T[d, r]   = sum_tok V[tok, d] P[tok, r]   A = V tile (MN-major, 128B swizzle, straight from TMA)
//                                              B = P^T    (MN-major, no swizzle, 16-byte stores per thread)
// so one HBM pass over each KV block serves every q head of its group and every draft position.
//
// Work split: every CTA is persistent (one per SM) and owns a cost-weighted share of the 128-token tiles of all
// (sequence, kv head) segments, in (sequence, kv head, tile) order.  A segment inside one CTA is finished there;
// one cut by a CTA boundary leaves a normalised partial + log2-sum-exp per piece, and the last piece to finish
// (counted with an atomic ticket) merges them all in the same launch.
// The split depends only on the batch's lengths (padding sequences of length 0 change nothing), and there is no
// host value or device read-back involved: graph-capturable with a fixed launch geometry.
//
// Warp roles (256 threads; 384 for the 32/48-row instantiations):
//   0 = K producer, 3 = V producer: block-table ids prefetched 32 tiles at a time, then TMA 64 dims x 128 tokens
//       boxes into rings (3 stages at 16 rows, 2 at 32/48); K slots are released right after S = K Q^T, V slots
//       after the PV product.  They start before the TMEM allocation and leave when done; the other warps meet on
//       named barrier 3;
//   1 = TMEM owner + UMMA issuer: products in a fixed order, QK(0), QK(1), then PV(j), QK(j+2), ... (S and P
//       buffers, and O except in the speculative-weights variant, are reused by tile parity, so this order is what
//       keeps every barrier within one phase);
//   2 = Q loader: gathers a segment's rows into the swizzled operand layout (cp.async, zero-filled padding);
//   4..7 (and 8..11) = softmax: thread ct of a warpgroup owns TMEM lane ct (token ct of S^T, dim ct of O^T).
//       Column maxima and sums over the 128 tokens use a transposed butterfly (each shuffle stage halves the rows
//       a lane carries).  With two warpgroups each takes half of the rows; rows never interact in the softmax.
//
// Fixed-length batches of 33-48 rows (verify with 8 or more drafts) run a speculative-weights variant of the 48-row
// instantiation: unscaled scores, no mask on tiles every row sees in full, the weights taken before the rescale vote
// (packed FP32) and voted on by their sum, and the O accumulator kept in TMEM across a segment's tiles.
#include <type_traits>

#include "nva_ptx.cuh"
#include "nva_kernels.h"

namespace nva {

namespace {

constexpr int kSlab = 128 * 128;        // 128 rows x 128 bytes (64 bf16 dims)
constexpr int kTileBytes = 2 * kSlab;   // one K or V tile: dims 0-63 and 64-127
constexpr int kConsumerBase = 128;
constexpr float kNegInf = -__builtin_huge_valf();
constexpr uint32_t kFull = 0xffffffffu;
// Tile descriptors travel from the K producer to the MMA and softmax warps through a ring of this depth.  The
// producer runs at most Cfg::kKStages (<= 3) tiles ahead of the S products and those at most 2 ahead of the softmax
// warps, so an entry is never rewritten before the softmax warps have read it.
constexpr int kInfoRing = 8;

constexpr int kMergePieces = 16;   // pieces of a cut segment merged through the shared weight table
constexpr int kTicketStride = 4;   // merge tickets per CTA: one per softmax warpgroup (at most 3)
// Row maxima move only when a score passes them by more than this (log2 units): until then P <= 2^8, exact enough in
// bf16 and in the FP32 sums.
constexpr float kRescaleLog2 = 8.0f;
constexpr float kRescaleSum = 256.0f;   // 2^kRescaleLog2: a thread's weights adding up to this ask for the exact maxima

template <int NP, bool Spec = false>
struct Cfg {
  static_assert(!Spec || NP == 48, "the speculative-weights variant is a 48-row instantiation");
  // softmax warpgroups (row shares): two at 32/48 rows.  Three at 48 rows measured 69 vs 72 us on verify k = 8 but
  // 216 vs 210 us on config 4's mixed step (short segments leave two groups idle; 128 registers a thread spill)
  static constexpr int kWG = NP >= 32 ? 2 : 1;
  static constexpr int kThreads = kConsumerBase + 128 * kWG;
  static constexpr int kRowsPerGroup = NP / kWG;                 // per-thread row arrays
  // Ring depths: 3 tiles; 2 for the 32/48-row tiles, whose softmax needs longer per tile than HBM does and whose
  // second Q buffer needs the room (a third V stage there measured slightly slower: 228 vs 221 us on config 4)
  static constexpr int kKStages = NP >= 32 ? 2 : 3;
  static constexpr int kVStages = NP >= 32 ? 2 : 3;
  static constexpr int kQBuf = 2;                                // Q double buffer: next segment's rows load early
  // P^T / O buffers: two at 32/48 rows, so a tile's P is handed to the tensor pipe before the previous tile's O is
  // folded (verify k = 8 69.6 -> 65.5 us, mixed step 186 -> 181 us); one at 16 rows, where HBM sets the pace
  static constexpr int kPBuf = NP >= 32 ? 2 : 1;
  // Spec (the 48-row variant for fixed-length verify batches): the O accumulator stays in TMEM (PV(j) adds onto its
  // segment's O; two O buffers, by segment parity), so the softmax warps touch O only at a segment's end and when a
  // tile moves some row maxima (scaled by alpha before PV(j) adds on); and the weights are taken before the rescale
  // vote, against the running maxima, their per-thread sum deciding the vote.  Otherwise each PV(j) is written fresh
  // and folded into registers, and the vote compares scores with the maxima first.
  static constexpr bool kOAcc = Spec;
  static constexpr bool kSpec = Spec;
  static constexpr int kK = 0;                                   // K ring
  static constexpr int kV = kKStages * kTileBytes;               // V ring
  static constexpr int kQ = (kKStages + kVStages) * kTileBytes;  // Q buffers, NP * 256 bytes each
  static constexpr int kP = kQ + kQBuf * NP * 256;               // [kPBuf] P^T, NP * 256 bytes each
  static constexpr int kBarCount = kPBuf == 2 ? 33 : 31;         // mbarriers (the B_* enum)
  static constexpr int kBars = kP + kPBuf * NP * 256;            // kBarCount x u64
  static constexpr int kInfo = kBars + (kBarCount * 8 + 15) / 16 * 16;   // kInfoRing x 2 x int4
  static constexpr int kRed = kInfo + kInfoRing * 32;            // [2][4][NP] column maxima per warp
  static constexpr int kM = kRed + 2 * 4 * NP * 4;               // [NP] running max (log2 units)
  static constexpr int kNegM = kM + NP * 4;                      // (kSpec) [NP] its negation, 0 for -inf
  static constexpr int kAlpha = kNegM + (kSpec ? NP * 4 : 0);    // [2][NP] rescale factors
  static constexpr int kLred = kAlpha + 2 * NP * 4;              // [4][NP] column sums per warp
  static constexpr int kRowOut = kLred + 4 * NP * 4;             // [NP] per-row output offset (int64)
  static constexpr int kRowInv = kRowOut + NP * 8;               // [NP] per-row 1 / sum
  static constexpr int kMergeW = kRowInv + NP * 4;               // [kWG][NP][kMergePieces] merge weights
  static constexpr int kTmem = kMergeW + kWG * NP * kMergePieces * 4;
  static constexpr int kAbort = kTmem + 4;
  static constexpr int kScan = (kAbort + 4 + 7) & ~7;            // [16] int2 per-warp prefix totals
  static constexpr int kPrefix = kScan + 16 * 8;                 // [kMaxDecodeSeqs + 1] tiles
  static constexpr int kCPrefix = kPrefix + (kMaxDecodeSeqs + 1) * 4;   // [kMaxDecodeSeqs + 1] cost units
  static constexpr int kEnd = kCPrefix + (kMaxDecodeSeqs + 1) * 4;
  static constexpr int kBytes = kEnd + 1024;                     // + slack for 1024-byte alignment
};

// S is double buffered by tile parity (S(j) in buffer j & 1); P by tile parity when Cfg::kPBuf = 2 (P(j) in buffer
// j & 1, with O in buffer (segment parity) accumulated over the segment's tiles), else single (buffer 0, O(j) =
// P(j) V(j) written fresh).  The barriers of P buffer b: pfull_bar(b), and ofull_bar(b) (completes when the PV
// product that read P buffer b finished); buffer 1's come last, so one-buffer instantiations keep a 31-barrier area.
enum {
  B_KFULL = 0, B_KEMPTY = 3, B_VFULL = 6, B_VEMPTY = 9, B_SFULL = 12, B_SEMPTY = 14, B_PFULL = 16, B_OFULL = 17,
  B_QFULL = 18, B_QEMPTY = 20, B_INFO = 22,   // B_INFO + kInfoRing <= B_KSTART
  B_KSTART = 30,  // the K producer has issued its first tile (the V producer starts after it)
  B_PFULL1 = 31, B_OFULL1 = 32
};
static_assert(B_PFULL1 - B_PFULL == B_OFULL1 - B_OFULL, "buffer 1's barriers at one distance");
__device__ __forceinline__ int pfull_bar(int b) { return B_PFULL + b * (B_PFULL1 - B_PFULL); }
__device__ __forceinline__ int ofull_bar(int b) { return B_OFULL + b * (B_OFULL1 - B_OFULL); }

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

// Cost of a (sequence, kv head) segment in the work split, in tile units: its tiles plus this much for the segment's
// start and end (Q load, first-tile latency, final PV, normalisation, output, a merge).  Fitted on B200 from per-CTA
// finish times at 1.8 (decode) to 3 (verify) tiles; 3 measured best on verify and mixed steps and neutral on decode.
constexpr int kSegCost = 3;

// Exclusive prefix sums over the sequences, per kv head: prefix[b] = tiles before sequence b, cprefix[b] = cost units
// before it (tiles + kSegCost per non-empty segment; padding sequences add nothing).  Called by all `nthreads`
// threads of the block; ends with a __syncthreads.
__device__ void build_prefix(const DecodeParams& p, int* prefix, int* cprefix, int2* warp_tot, int tid,
                             int nthreads) {
  const int lane = tid & 31, warp = tid >> 5, nwarps = nthreads >> 5;
  int running = 0, crunning = 0;
  for (int base = 0; base < p.num_seqs; base += nthreads) {
    const int b = base + tid;
    const int v = b < p.num_seqs ? seq_tiles(p, b) : 0;
    const int cv = v > 0 ? v + kSegCost : 0;
    int x = v, cx = cv;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(kFull, x, o), cy = __shfl_up_sync(kFull, cx, o);
      if (lane >= o) {
        x += y;
        cx += cy;
      }
    }
    if (lane == 31) warp_tot[warp] = make_int2(x, cx);
    __syncthreads();
    int before = running, cbefore = crunning, chunk = 0, cchunk = 0;
    for (int w = 0; w < nwarps; ++w) {
      const int2 wt = warp_tot[w];
      if (w < warp) {
        before += wt.x;
        cbefore += wt.y;
      }
      chunk += wt.x;
      cchunk += wt.y;
    }
    if (b < p.num_seqs) {
      prefix[b] = before + x - v;
      cprefix[b] = cbefore + cx - cv;
    }
    running += chunk;
    crunning += cchunk;
    __syncthreads();
  }
  if (tid == 0) {
    prefix[p.num_seqs] = running;
    cprefix[p.num_seqs] = crunning;
  }
  __syncthreads();
}

struct Loc {
  int b, g, j, nt, s0;
};

// Cost-weighted split of the tiles over `grid` CTAs.  Tile j of segment (b, g) sits at cost position
// KVH * cprefix[b] + g * (nt + kSegCost) + kSegCost + j; CTA c owns the tiles whose positions fall in
// [c * per, (c + 1) * per), a contiguous range of global tile indices.  It depends only on the lengths.
struct Split {
  const int* prefix;
  const int* cprefix;
  int B, KVH, per, tiles;
  __device__ Split(const int* pf, const int* cpf, int nseq, int kvh, int grid) : prefix(pf), cprefix(cpf), B(nseq),
                                                                                KVH(kvh) {
    tiles = KVH * prefix[B];
    const int cost = KVH * cprefix[B];
    per = cost > 0 ? (cost + grid - 1) / grid : 1;
  }
  __device__ int pos(int b, int g, int j) const {
    const int nt = prefix[b + 1] - prefix[b];
    return KVH * cprefix[b] + g * (nt + kSegCost) + kSegCost + j;
  }
  __device__ int owner(int b, int g, int j) const { return pos(b, g, j) / per; }
  // first global tile index of CTA c (tiles when c owns nothing further)
  __device__ int begin(int c) const {
    const int x = c * per;
    if (x >= KVH * cprefix[B]) return tiles;
    int lo = 0, hi = B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (KVH * cprefix[mid] <= x) lo = mid; else hi = mid - 1;
    }
    const int nt = prefix[lo + 1] - prefix[lo];
    const int rem = x - KVH * cprefix[lo];
    const int g = rem / (nt + kSegCost);
    const int o = rem - g * (nt + kSegCost);
    return KVH * prefix[lo] + g * nt + max(0, o - kSegCost);
  }
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

// Transposed butterfly over the 32 lanes of a warp for NR (power of two <= 32) columns held by every lane: each
// stage sends half of the remaining columns to the partner lane and keeps the other half, so the whole reduction
// costs NR - 1 + (5 - log2 NR) shuffles with the shuffles of a stage independent of each other.  On return lane l
// holds the reduction of column l / (32 / NR) in v[0]; lanes with l % (32 / NR) == 0 store it to dst[column].
template <int N, int O, bool kMax>
__device__ __forceinline__ void column_stage(float* v, int lane) {
  if constexpr (O > 0) {
    if constexpr (N > 1) {
      constexpr int H = N / 2;
      const bool upper = (lane & O) != 0;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const float send = upper ? v[i] : v[i + H];
        const float keep = upper ? v[i + H] : v[i];
        const float recv = __shfl_xor_sync(kFull, send, O);
        v[i] = kMax ? fmaxf(keep, recv) : keep + recv;
      }
      column_stage<H, O / 2, kMax>(v, lane);
    } else {
      const float recv = __shfl_xor_sync(kFull, v[0], O);
      v[0] = kMax ? fmaxf(v[0], recv) : v[0] + recv;
      column_stage<1, O / 2, kMax>(v, lane);
    }
  }
}

template <int NR, bool kMax>
__device__ __forceinline__ void column_reduce(float* v, float* dst, int lane) {
  column_stage<NR, 16, kMax>(v, lane);
  constexpr int kRep = 32 / NR;
  if ((lane & (kRep - 1)) == 0) dst[lane / kRep] = v[0];
}

// Column reduction of NR (8, 16, 24, 32 or 48) values per thread within one warp into dst[0..NR).
template <int NR, bool kMax>
__device__ __forceinline__ void warp_columns(const float* x, float* dst, int lane) {
  float v[32];
  if constexpr (NR <= 16) {
#pragma unroll
    for (int i = 0; i < NR; ++i) v[i] = x[i];
    column_reduce<NR, kMax>(v, dst, lane);
  } else if constexpr (NR == 24) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = x[i];
    column_reduce<16, kMax>(v, dst, lane);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = x[16 + i];
    column_reduce<8, kMax>(v, dst + 16, lane);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = x[i];
    column_reduce<32, kMax>(v, dst, lane);
    if constexpr (NR == 48) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = x[32 + i];
      column_reduce<16, kMax>(v, dst + 32, lane);
    }
  }
}

// Rows a segment carries through the softmax: its real rows rounded up to 8, 16, 32 or 48 (never above NP).
__device__ __forceinline__ int rows_width(int R) { return R <= 8 ? 8 : R <= 16 ? 16 : R <= 32 ? 32 : 48; }
// UMMA N for a segment (M = 128 needs N to be a multiple of 16).
__device__ __forceinline__ int mma_width(int R) { return R <= 16 ? 16 : R <= 32 ? 32 : 48; }

// Calls f(integral_constant<NR>) for the row width nr, limited to the kernel's NP.
template <int NP, class F>
__device__ __forceinline__ void with_rows(int nr, F&& f) {
  if (nr <= 8) {
    f(std::integral_constant<int, 8>{});
  } else if (nr <= 16 || NP == 16) {
    f(std::integral_constant<int, 16>{});
  } else if (nr <= 32 || NP == 32) {
    f(std::integral_constant<int, (NP >= 32 ? 32 : 16)>{});
  } else {
    f(std::integral_constant<int, NP>{});
  }
}

// The UMMA issuing lane, by row tile (measured on B200 against a softmax warp on the issuer's SM sub-partition):
// elect.sync for 32/48-row tiles (verify k = 8 about 6% faster), a fixed lane 0 for the 16-row decode tile (about
// 2% faster there).
template <int NP>
__device__ __forceinline__ bool umma_lane(int lane) {
  if constexpr (NP >= 32) {
    return elect_one();
  } else {
    return lane == 0;
  }
}

// Rows each of `wg_count` softmax warpgroups carries for an NR-wide tile: all NR with one group; otherwise NR split
// into equal shares rounded up to whole 8-row P^T vectors (8, 16 or 24 rows); groups past NR hold padding only.
__host__ __device__ constexpr int group_rows_rt(int wg_count, int nr) {
  return wg_count == 1 ? nr : nr <= 8 ? 8 : ((nr + wg_count - 1) / wg_count + 7) / 8 * 8;
}

// The same at compile time, for the kernel's group count.
template <int NP, int NR>
__device__ __forceinline__ constexpr int group_rows() {
  return group_rows_rt(Cfg<NP>::kWG, NR);
}

// HR consecutive TMEM columns (8, 16 or 24) of this warp's lanes, one wait.
template <int HR>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float* v) {
  if constexpr (HR == 8) {
    tmem_ld8(taddr, v);
  } else if constexpr (HR == 16) {
    tmem_ld16(taddr, v);
  } else {
    static_assert(HR == 24, "row group width");
    tmem_ld24(taddr, v);
  }
}

// Merge the pieces of a cut segment (CTAs c0..c1) into its output rows [r0, r1), from one 128-thread group (all of
// its threads call this; named barrier bar_id).  Each piece is weighted by 2^(lse - max lse) / sum.  The partials were
// written by other CTAs, so they are read past L1 (ld.global.cg).  Two pieces: (row, 4 dims) items six at a time
// with all their loads in one round.  Up to kMergePieces pieces: one thread per row puts the row's weights in the
// group's table `wsm`, then items four at a time (two memory rounds).  More pieces: a plain loop.
template <int NP>
__device__ __forceinline__ void merge_pieces(const DecodeParams& p, int c0, int c1, int r0, int r1, int G,
                                             int64_t out_base, int ct, float* wsm, uint32_t bar_id) {
  const int pieces = c1 - c0 + 1;
  auto slot_of = [&](int pi) { return pi == 0 ? 2 * c0 + 1 : 2 * (c0 + pi); };
  auto store = [&](int idx, float4 a, float inv) {
    const int r = r0 + (idx >> 5), l4 = idx & 31;
    const int i = r / G, h = r - i * G;
    uint2 packed;
    packed.x = pack_bf16x2(a.x * inv, a.y * inv);
    packed.y = pack_bf16x2(a.z * inv, a.w * inv);
    *reinterpret_cast<uint2*>(p.out + out_base + (int64_t)i * p.out_row_stride + h * kHeadDim + l4 * 4) = packed;
  };
  if (pieces == 2) {
    // a segment cut once (the usual case): every load of a round of six items issued together
    const int s0 = 2 * c0 + 1, s1 = 2 * c0 + 2;
    const int nitems = (r1 - r0) * 32;
    constexpr int kRound = 2;
    for (int base = ct; base < nitems; base += kRound * 128) {
      float4 a0[kRound], a1[kRound];
      float e0[kRound], e1[kRound];
#pragma unroll
      for (int u = 0; u < kRound; ++u) {
        const int idx = base + u * 128;
        if (idx < nitems) {
          const int r = r0 + (idx >> 5), l4 = idx & 31;
          e0[u] = __ldcg(p.part_lse + s0 * NP + r);
          e1[u] = __ldcg(p.part_lse + s1 * NP + r);
          a0[u] = __ldcg(reinterpret_cast<const float4*>(p.part_o + ((int64_t)s0 * NP + r) * kHeadDim) + l4);
          a1[u] = __ldcg(reinterpret_cast<const float4*>(p.part_o + ((int64_t)s1 * NP + r) * kHeadDim) + l4);
        }
      }
#pragma unroll
      for (int u = 0; u < kRound; ++u) {
        const int idx = base + u * 128;
        if (idx < nitems) {
          const float mx = fmaxf(e0[u], e1[u]);
          const float w0 = (mx == kNegInf || e0[u] == kNegInf) ? 0.f : fast_exp2(e0[u] - mx);
          const float w1 = (mx == kNegInf || e1[u] == kNegInf) ? 0.f : fast_exp2(e1[u] - mx);
          const float den = w0 + w1;
          const float4 acc = make_float4(w0 * a0[u].x + w1 * a1[u].x, w0 * a0[u].y + w1 * a1[u].y,
                                         w0 * a0[u].z + w1 * a1[u].z, w0 * a0[u].w + w1 * a1[u].w);
          store(idx, acc, den > 0.f ? 1.f / den : 0.f);
        }
      }
    }
    return;
  }
  if (pieces <= kMergePieces) {
    for (int r = r0 + ct; r < r1; r += 128) {
      float* w = wsm + (r - r0) * kMergePieces;
      float mx = kNegInf;
      for (int pi = 0; pi < pieces; ++pi) {
        const float v = __ldcg(p.part_lse + slot_of(pi) * NP + r);
        w[pi] = v;
        mx = fmaxf(mx, v);
      }
      float den = 0.f;
      for (int pi = 0; pi < pieces; ++pi) {
        const float e = (mx == kNegInf || w[pi] == kNegInf) ? 0.f : fast_exp2(w[pi] - mx);
        w[pi] = e;
        den += e;
      }
      const float inv = den > 0.f ? 1.f / den : 0.f;
      for (int pi = 0; pi < pieces; ++pi) w[pi] *= inv;
    }
    named_bar_sync(bar_id, 128);
    const int nitems = (r1 - r0) * 32;
    for (int base = ct; base < nitems; base += 4 * 128) {
      float4 acc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int idx = base + u * 128;
        if (idx < nitems) {
          const int r = r0 + (idx >> 5), l4 = idx & 31;
          const float* w = wsm + (r - r0) * kMergePieces;
          for (int pi = 0; pi < pieces; ++pi) {
            const float4 v =
                __ldcg(reinterpret_cast<const float4*>(p.part_o + ((int64_t)slot_of(pi) * NP + r) * kHeadDim) + l4);
            const float wp = w[pi];
            acc[u].x += wp * v.x;
            acc[u].y += wp * v.y;
            acc[u].z += wp * v.z;
            acc[u].w += wp * v.w;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = base + u * 128;
        if (idx < nitems) store(idx, acc[u], 1.f);
      }
    }
    return;
  }
  for (int idx = ct; idx < (r1 - r0) * 32; idx += 128) {
    const int r = r0 + (idx >> 5), l4 = idx & 31;
    float mx = kNegInf;
    for (int pi = 0; pi < pieces; ++pi) mx = fmaxf(mx, __ldcg(p.part_lse + slot_of(pi) * NP + r));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float den = 0.f;
    if (mx != kNegInf) {
#pragma unroll 4
      for (int pi = 0; pi < pieces; ++pi) {
        const float lse = __ldcg(p.part_lse + slot_of(pi) * NP + r);
        const float4 v =
            __ldcg(reinterpret_cast<const float4*>(p.part_o + ((int64_t)slot_of(pi) * NP + r) * kHeadDim) + l4);
        const float w = lse == kNegInf ? 0.f : fast_exp2(lse - mx);
        acc.x += w * v.x;
        acc.y += w * v.y;
        acc.z += w * v.z;
        acc.w += w * v.w;
        den += w;
      }
    }
    store(idx, acc, den > 0.f ? 1.f / den : 0.f);
  }
}

template <int NP, bool Spec>
__global__ void __launch_bounds__(Cfg<NP, Spec>::kThreads, 1)
paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                    const DecodeParams p) {
  using C = Cfg<NP, Spec>;
  // P / O buffer of tile t and the phase parity of its barriers
  auto pbuf = [](int t) { return C::kPBuf == 2 ? (t & 1) : 0; };
  auto pphase = [](int t) { return C::kPBuf == 2 ? ((t >> 1) & 1) : (t & 1); };
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBars);
  int4* info = reinterpret_cast<int4*>(smem + C::kInfo);       // [kInfoRing][2]
  float* red = reinterpret_cast<float*>(smem + C::kRed);
  float* m_s = reinterpret_cast<float*>(smem + C::kM);
  float* negm_s = reinterpret_cast<float*>(smem + C::kNegM);
  float* alpha_s = reinterpret_cast<float*>(smem + C::kAlpha);
  float* lred = reinterpret_cast<float*>(smem + C::kLred);
  int64_t* row_out = reinterpret_cast<int64_t*>(smem + C::kRowOut);
  float* row_inv = reinterpret_cast<float*>(smem + C::kRowInv);
  float* merge_w = reinterpret_cast<float*>(smem + C::kMergeW);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kTmem);
  volatile int* abort = reinterpret_cast<volatile int*>(smem + C::kAbort);
  int2* warp_tot = reinterpret_cast<int2*>(smem + C::kScan);
  int* prefix = reinterpret_cast<int*>(smem + C::kPrefix);
  int* cprefix = reinterpret_cast<int*>(smem + C::kCPrefix);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int KVH = p.num_kv_heads;
  const int G = p.group;

  if (tid == 0) {
    for (int s = 0; s < C::kKStages; ++s) {
      mbar_init(&bars[B_KFULL + s], 1);
      mbar_init(&bars[B_KEMPTY + s], 1);
    }
    for (int s = 0; s < C::kVStages; ++s) {
      mbar_init(&bars[B_VFULL + s], 1);
      mbar_init(&bars[B_VEMPTY + s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[B_SFULL + i], 1);
      mbar_init(&bars[B_SEMPTY + i], 128 * C::kWG);
      mbar_init(&bars[B_QFULL + i], 32);
      mbar_init(&bars[B_QEMPTY + i], 1);
    }
    for (int i = 0; i < C::kPBuf; ++i) {
      mbar_init(&bars[pfull_bar(i)], 128 * C::kWG);
      mbar_init(&bars[ofull_bar(i)], 1);
    }
    for (int i = 0; i < kInfoRing; ++i) mbar_init(&bars[B_INFO + i], 1);
    mbar_init(&bars[B_KSTART], 1);
    *abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  // With a programmatic dependency on the preceding kernel (the prefill plan of a varlen call): everything above ran
  // beside its end; wait for it before the first global read, then let the next grid (the call's prefill kernel)
  // start its blocks.
  if (p.pdl) {
    griddep_wait();
    if (tid == 0) griddep_launch_dependents();
  }
  build_prefix(p, prefix, cprefix, warp_tot, tid, C::kThreads);   // ends with __syncthreads
  // sequences whose query rows see no key (length 0: batch padding) get zero rows, from CTA b % grid
  for (int b = blockIdx.x; b < p.num_seqs; b += gridDim.x) {
    const SeqShape ss = seq_shape(p, b);
    if (ss.n >= 1 && ss.n <= p.max_n && ss.L < 1) {
      const int per_row = p.num_heads * kHeadDim;
      for (int idx = tid; idx < ss.n * per_row; idx += C::kThreads) {
        const int i = idx / per_row, rem = idx - i * per_row;
        p.out[(int64_t)(ss.q0 + i) * p.out_row_stride + rem] = __float2bfloat16_rn(0.f);
      }
    }
  }

  const Split split(prefix, cprefix, p.num_seqs, KVH, gridDim.x);
  const int t_begin = split.begin(blockIdx.x);
  const int t_end = split.begin(blockIdx.x + 1);
  const int ntiles = t_end > t_begin ? t_end - t_begin : 0;
  if (ntiles == 0) return;   // nothing for this CTA (e.g. a varlen batch without short runs): no TMEM, no pipeline
  if (warp == 0 || warp == 3) {
    // ------------------------------------------------------------ K (warp 0) and V (warp 3) producers
    // They need no TMEM and start streaming at once; they leave when their tiles are issued (the other warps wait
    // for every tile, so the block outlives the copies).  K goes first: the V producer starts after the first K tile
    // is issued, so that across the GPU the first S products are not queued behind V tiles needed later.
    const bool is_k = warp == 0;
    const CUtensorMap* tm = is_k ? &tm_k : &tm_v;
    uint8_t* ring = smem + (is_k ? C::kK : C::kV);
    uint64_t* full = bars + (is_k ? B_KFULL : B_VFULL);
    uint64_t* empty = bars + (is_k ? B_KEMPTY : B_VEMPTY);
    const int stages = is_k ? C::kKStages : C::kVStages;
    bool stop = !is_k && !mbar_wait_warp(&bars[B_KSTART], 0, abort);
    for (int base = 0; base < ntiles && !stop; base += 32) {
      // lane-parallel descriptors of the next 32 tiles (the block-table reads overlap each other)
      int g = 0, j = 0, b = 0, row0 = 0, flags = 0, n = 0, L = 0, q0 = 0, nt = 0;
      if (base + lane < ntiles) {
        const int t = t_begin + base + lane;
        const Loc lc = locate(t, prefix, p.num_seqs, KVH);
        b = lc.b;
        g = lc.g;
        j = lc.j;
        nt = lc.nt;
        const int tok0 = j * kTileTokens;
        int page = __ldg(p.block_tables + (int64_t)b * p.bt_stride + tok0 / p.block_size);
        if (page < 0 || page >= p.num_blocks) {
          if (is_k) atomicOr(&g_error_word, kErrBlockRange);
          page = -1;   // TMA fills out-of-range rows with zeros; nothing outside the pool is read
        }
        row0 = page * p.block_size + (tok0 % p.block_size);
        flags = (j == 0 || t == t_begin ? 1 : 0) | (j == nt - 1 || t == t_end - 1 ? 2 : 0);
        if (is_k) {
          const SeqShape ss = seq_shape(p, b);
          n = ss.n;
          L = ss.L;
          q0 = ss.q0;
        }
      }
      const int cnt = min(32, ntiles - base);
      for (int i = 0; i < cnt; ++i) {
        const int jj = base + i;
        const int st = jj % stages;
        const int gi = __shfl_sync(kFull, g, i), ri = __shfl_sync(kFull, row0, i);
        const int bi = __shfl_sync(kFull, b, i), ji = __shfl_sync(kFull, j, i), fi = __shfl_sync(kFull, flags, i);
        const int ni = __shfl_sync(kFull, n, i), Li = __shfl_sync(kFull, L, i), qi = __shfl_sync(kFull, q0, i);
        const int nti = __shfl_sync(kFull, nt, i);
        if (!mbar_wait_warp(&empty[st], ((jj / stages) & 1) ^ 1, abort)) {
          stop = true;
          break;
        }
        if (elect_one()) {
          if (is_k) {
            const int e = jj % kInfoRing;
            info[2 * e] = make_int4(bi, gi, ji, fi);
            info[2 * e + 1] = make_int4(ni, Li, qi, nti);
            mbar_arrive(&bars[B_INFO + e]);
          }
          mbar_arrive_expect_tx(&full[st], kTileBytes);
          uint8_t* dst = ring + st * kTileBytes;
          tma_load_3d(dst, tm, 0, gi, ri, &full[st]);
          tma_load_3d(dst + kSlab, tm, 64, gi, ri, &full[st]);
          if (is_k && jj == 0) mbar_arrive(&bars[B_KSTART]);
        }
        __syncwarp();
      }
    }
    return;
  }
  // ------------------------------------------------------------ the other warps: TMEM, then their roles
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  named_bar_sync(3, C::kThreads - 64);
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 1 && ntiles > 0) {
    // ------------------------------------------------------------ UMMA issuer (whole warp polls, an elected lane issues)
    const uint64_t q_desc0 = umma_desc_sw128(smem_u32(smem + C::kQ), 16, 1024);
    const uint64_t k_desc0 = umma_desc_sw128(smem_u32(smem + C::kK), 16, 1024);
    const uint64_t v_desc0 = umma_desc_sw128(smem_u32(smem + C::kV), kSlab, 1024);
    const uint64_t p_desc0 = umma_desc_noswz(smem_u32(smem + C::kP), 128, 2048);
    // Issue order: QK(0), QK(1), then PV(j), QK(j+2), ...  The softmax warps find S(j+1) ready when they finish
    // tile j, and every wait is a blocking, hardware-suspended mbarrier wait (no polling next to a softmax warp).
    int qk = 0, pv = 0, qseg = 0;
    bool ok = true;
    auto issue_qk = [&]() {
      if (!ok || qk >= ntiles) return;
      const int st = qk % C::kKStages;
      const int e = qk % kInfoRing;
      if (!mbar_wait_warp(&bars[B_KFULL + st], (qk / C::kKStages) & 1, abort)) { ok = false; return; }
      const int flags = info[2 * e].w;
      // UMMA N for this tile's segment: its rows rounded up to 16/32/48
      const uint32_t idesc_qk = umma_idesc_bf16(128, min(NP, mma_width(info[2 * e + 1].x * G)), false, false);
      const int qb = qseg % C::kQBuf;
      if ((flags & 1) && !mbar_wait_warp(&bars[B_QFULL + qb], (qseg / C::kQBuf) & 1, abort)) { ok = false; return; }
      const int buf = qk & 1;
      if (!mbar_wait_warp(&bars[B_SEMPTY + buf], ((qk >> 1) & 1) ^ 1, abort)) { ok = false; return; }
      tc_fence_after();
      if (umma_lane<NP>(lane)) {
        // K-major SW128 operands: step k at +32 B within a 128-byte row, steps 4..7 in the second slab
        constexpr uint32_t kOffK[8] = {0, 2, 4, 6, kSlab >> 4, (kSlab >> 4) + 2, (kSlab >> 4) + 4, (kSlab >> 4) + 6};
        constexpr uint32_t kOffQ[8] = {0, 2, 4, 6, (NP * 128) >> 4, ((NP * 128) >> 4) + 2, ((NP * 128) >> 4) + 4,
                                       ((NP * 128) >> 4) + 6};
        umma_bf16_ss_x8(tmem + buf * NP, k_desc0 + ((st * kTileBytes) >> 4), q_desc0 + ((qb * NP * 256) >> 4),
                        idesc_qk, 0u, kOffK, kOffQ);
        umma_commit(&bars[B_SFULL + buf]);
        umma_commit(&bars[B_KEMPTY + st]);
        if (flags & 2) umma_commit(&bars[B_QEMPTY + qb]);
      }
      __syncwarp();
      if (flags & 2) ++qseg;
      ++qk;
    };
    issue_qk();
    issue_qk();
    int oseg = 0;   // O buffer of the segment of tile pv (segment parity) when O accumulates in TMEM
    while (ok && pv < ntiles) {
      const int st = pv % C::kVStages;
      const int pb = pbuf(pv);   // P buffer of this tile
      if (!mbar_wait_warp(&bars[pfull_bar(pb)], pphase(pv), abort)) break;
      if (!mbar_wait_warp(&bars[B_VFULL + st], (pv / C::kVStages) & 1, abort)) break;
      const int e = pv % kInfoRing;
      const bool seg_first = C::kOAcc && (info[2 * e].w & 1);
      if (seg_first && pv > 0) oseg ^= 1;
      // O^T target and accumulate flag: the segment's accumulator (fresh at its first tile), or a fresh product
      const uint32_t o_col = C::kOAcc ? (2 + oseg) * NP : (2 + pb) * NP;
      const uint32_t o_acc = C::kOAcc && !seg_first ? 1u : 0u;
      const uint32_t idesc_pv = umma_idesc_bf16(128, min(NP, mma_width(info[2 * e + 1].x * G)), true, true);
      tc_fence_after();
      if (umma_lane<NP>(lane)) {
        // A = V^T: 16 tokens per step (two 8-row groups, SBO 1024; two 64-dim slabs, LBO 16 KB) -> +2048 B;
        // B = P^T: 16 tokens per step (two 8-token core-matrix groups, LBO 128; 8-row groups, SBO 2048) -> +256 B
        constexpr uint32_t kOffV[8] = {0, 128, 256, 384, 512, 640, 768, 896};
        constexpr uint32_t kOffP[8] = {0, 16, 32, 48, 64, 80, 96, 112};
        umma_bf16_ss_x8(tmem + o_col, v_desc0 + ((st * kTileBytes) >> 4), p_desc0 + ((pb * NP * 256) >> 4),
                        idesc_pv, o_acc, kOffV, kOffP);
        umma_commit(&bars[ofull_bar(pb)]);
        umma_commit(&bars[B_VEMPTY + st]);
      }
      __syncwarp();
      ++pv;
      issue_qk();
    }
  } else if (warp == 2 && ntiles > 0) {
    // ------------------------------------------------------------ Q loader
    int qi = 0;
    int t = t_begin;
    while (t < t_end) {
      const Loc lc = locate(t, prefix, p.num_seqs, KVH);
      const int qb = qi % C::kQBuf;
      if (!mbar_wait_warp(&bars[B_QEMPTY + qb], ((qi / C::kQBuf) & 1) ^ 1, abort)) break;
      const SeqShape ss = seq_shape(p, lc.b);
      const int R = ss.n * G;
      const int rows = min(NP, mma_width(R));   // the rows the S product reads; those past R are zero
      uint8_t* qs = smem + C::kQ + qb * NP * 256;
      for (int idx = lane; idx < rows * 16; idx += 32) {
        const int r = idx >> 4, c = idx & 15;
        const int rr = r < R ? r : 0;
        const int i = rr / G, h = rr - i * G;
        const __nv_bfloat16* src =
            p.q + (int64_t)(ss.q0 + i) * p.q_row_stride + (int64_t)(lc.g * G + h) * kHeadDim + c * 8;
        cp_async_16(qs + (c >> 3) * (NP * 128) + sw128_offset(r, c & 7), src, r < R ? 16u : 0u);
      }
      cp_async_wait_all();
      fence_proxy_async_smem();
      __syncwarp();
      mbar_arrive(&bars[B_QFULL + qb]);
      ++qi;
      t = lc.s0 + lc.nt;   // next segment
    }
  } else if (warp >= 4 && ntiles > 0) {
    // ------------------------------------------------------------ softmax / accumulation
    // Warpgroup wg owns rows [rb, rb + HR) of the segment's NR-wide tile (all rows when there is one group).  The
    // groups share nothing but the S / P / O buffers' barriers: each has its own named barrier (1 + wg) and its
    // own rows of the shared row arrays.  Every wait here is warp-uniform and every named barrier ORs "gave up"
    // across the group's four warps, so they leave the loop together if a wait expires; the barrier sequence is
    // the same for every row width, so a warp that gave up still matches the others.
    const int cidx = tid - kConsumerBase;
    const int ct = cidx & 127;                // TMEM lane: token ct of S^T, dim ct of O^T
    const int wg = cidx >> 7;
    const int wq = ct >> 5;                   // lane quadrant
    const uint32_t bar_id = 1 + wg;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    uint8_t* p_smem = smem + C::kP;
    constexpr int NPH = C::kRowsPerGroup;
    float l[NPH], o[NPH], s[NPH];
    int R = 0, nr = 8, n = 0, L = 0, q0 = 0, seg_s0 = 0, seg_s1 = 0, seg_g = 0, seg_b = 0;
    bool alive = true;
    bool rescaled_prev = false;               // whether the previous tile moved some row maxima (alpha != 1)
    int ob = 0;                               // O accumulator of the current segment (Cfg::kOAcc): segment parity
    // A piece of a cut segment is done (this group's rows [rb, rb + hr) written): take the group's ticket for the
    // segment; the group that brings it to the number of pieces merges those rows of all pieces and puts the
    // counter back to zero, so the counters are zero again when the launch ends (the workspace contract).  Every
    // thread of the group calls this.
    auto arrive_and_merge = [&](int c0, int c1, int rb_, int hr_) {
      named_bar_sync(bar_id, 128);
      bool last_arrival = false;
      if (ct == 0) {
        int32_t* ticket = p.counters + kTicketStride * c0 + wg;
        __threadfence();   // release: the group's partial rows (ordered before by the barrier) before the ticket
        last_arrival = atomicAdd(ticket, 1) == c1 - c0;
        if (last_arrival) {
          __threadfence();   // acquire: the other pieces' rows, for the whole group after the barrier below
          *ticket = 0;
        }
      }
      if (named_bar_any(bar_id, 128, last_arrival))
        merge_pieces<NP>(p, c0, c1, rb_, min(rb_ + hr_, R), G,
                         (int64_t)q0 * p.out_row_stride + (int64_t)seg_g * G * kHeadDim, ct,
                         merge_w + wg * NP * kMergePieces, bar_id);
    };
    for (int jj = 0; jj < ntiles; ++jj) {
      const int st = jj % C::kVStages;      // V ring slot of this tile
      const int buf = jj & 1;
      const int e = jj % kInfoRing;
      alive = alive && mbar_wait_warp(&bars[B_INFO + e], (jj / kInfoRing) & 1, abort);
      int4 inf = make_int4(0, 0, 0, 0);
      if (alive) inf = info[2 * e];
      const bool first = inf.w & 1, last = inf.w & 2;
      if (C::kOAcc && first && jj > 0) ob ^= 1;
      if (alive && first) {
        const int4 sh = info[2 * e + 1];
        n = sh.x;
        L = sh.y;
        q0 = sh.z;
        seg_g = inf.y;
        seg_b = inf.x;
        R = n * G;
        nr = min(NP, rows_width(R));
        seg_s0 = KVH * prefix[inf.x] + seg_g * sh.w;
        seg_s1 = seg_s0 + sh.w;
#pragma unroll
        for (int r = 0; r < NPH; ++r) {
          l[r] = 0.f;
          if constexpr (!C::kOAcc) o[r] = 0.f;   // (in TMEM, O starts fresh with the segment's first PV)
        }
      }
      const int hr = group_rows_rt(C::kWG, nr);
      const int rb = wg * hr;
      const int tok0 = inf.z * kTileTokens;
      const int tok = tok0 + ct;
      if (C::kWG > 1 && rb >= R) {
        // every row of this group is padding (a short segment): only keep the S / P phases paced.  SEMPTY of
        // tile jj is given after S(jj) exists and PFULL of jj after PV(jj-2) (the buffer's last product) finished,
        // as the working group does, so no arrival can land in a phase that the other group has not reached.
        alive = alive && mbar_wait_warp(&bars[B_SFULL + buf], (jj >> 1) & 1, abort);
        if (alive) mbar_arrive(&bars[B_SEMPTY + buf]);
        // (two groups: always two P buffers)
        if (jj >= 2) alive = alive && mbar_wait_warp(&bars[ofull_bar(pbuf(jj))], pphase(jj - 2), abort);
        if (alive) mbar_arrive(&bars[pfull_bar(pbuf(jj))]);
        // A warp whose descriptor wait gave up decides padding vs working rows from the previous segment's R, so on
        // the way out this path mirrors the working path's two votes (the rescale vote, then the "gave up" vote):
        // whichever path each warp of the group took, their barrier arrivals pair up and all leave together.
        if (named_bar_any(bar_id, 128, !alive)) {
          named_bar_any(bar_id, 128, true);
          break;
        }
        continue;
      }
      // ---- S tile -> weights.  Row maxima are lazy: the weights P = 2^(s * scale - m) are taken against each row's
      // running maximum m, and the exact tile maxima (per-warp column maxima -> row owners) only at a segment's
      // first tile and when some weight could reach 2^kRescaleLog2; otherwise alpha = 1 and the reduction and two
      // barriers are skipped.  Either way every weight stays below 2^kRescaleLog2.
      //   kSpec (48 rows): the weights come first (packed FP32 pairs) and a thread whose weights add up to
      //   2^kRescaleLog2 votes for the exact path, which loads the unscaled scores again (the S buffer is released
      //   after the vote) and takes the weights against the new maxima.  Tiles that every row sees in full skip the
      //   mask: rows past R (up to the UMMA N) hold zero scores there, from the zero-filled Q rows, and weigh nothing
      //   (offset -128).
      //   Otherwise: scores are masked and scaled, the vote compares them with m + 2^kRescaleLog2, and the weights
      //   follow it.
      alive = alive && mbar_wait_warp(&bars[B_SFULL + buf], (jj >> 1) & 1, abort);
      bool need = first;
      const bool open_tile = C::kSpec && tok0 + kTileTokens - 1 <= L - n;
      // query i of the segment sees tokens <= L - n + i, i.e. row r = i*G + h is visible iff r >= G*(tok-L+n)
      const int d = tok - (L - n);
      const int rmin = d > 0 ? d * G : 0;
      auto load_scores = [&](auto hr_c) {   // (kSpec) unscaled scores, masked unless the tile is open
        constexpr int HR = decltype(hr_c)::value;
        tmem_ld_cols<HR>(t_lane + buf * NP + rb, s);
        if (!open_tile) {
#pragma unroll
          for (int i = 0; i < HR; ++i) {
            const int r = rb + i;
            s[i] = (r >= rmin && r < R) ? s[i] : kNegInf;
          }
        }
      };
      auto weights = [&](auto hr_c) {   // (kSpec) s <- 2^(s * scale - m); returns the sum of this thread's weights
        constexpr int HR = decltype(hr_c)::value;
        const float* nm = negm_s + rb;
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
        float2 sum = make_float2(0.f, 0.f);
#pragma unroll
        for (int r = 0; r < HR; r += 4) {
          const float4 n4 = *reinterpret_cast<const float4*>(nm + r);
          const float2 x0 = ffma2(make_float2(s[r], s[r + 1]), sc2, make_float2(n4.x, n4.y));
          const float2 x1 = ffma2(make_float2(s[r + 2], s[r + 3]), sc2, make_float2(n4.z, n4.w));
          s[r] = fast_exp2(x0.x);
          s[r + 1] = fast_exp2(x0.y);
          s[r + 2] = fast_exp2(x1.x);
          s[r + 3] = fast_exp2(x1.y);
          sum = fadd2(sum, fadd2(make_float2(s[r], s[r + 1]), make_float2(s[r + 2], s[r + 3])));
        }
        return sum.x + sum.y;
      };
      if (alive) {
        tc_fence_after();
        with_rows<NP>(nr, [&](auto nr_c) {
          constexpr int HR = group_rows<NP, decltype(nr_c)::value>();
          if constexpr (C::kSpec) {
            load_scores(std::integral_constant<int, HR>{});
            if (!first) need = weights(std::integral_constant<int, HR>{}) >= kRescaleSum;
          } else {
            tmem_ld_cols<HR>(t_lane + buf * NP + rb, s);
            tc_fence_before();
            mbar_arrive(&bars[B_SEMPTY + buf]);
#pragma unroll
            for (int i = 0; i < HR; ++i) {
              const int r = rb + i;
              s[i] = (r >= rmin && r < R) ? s[i] * p.scale_log2 : kNegInf;
            }
            if (!first) {
              const float* ms = m_s + rb;
#pragma unroll
              for (int r = 0; r < HR; r += 4) {
                const float4 m4 = *reinterpret_cast<const float4*>(ms + r);
                need |= (s[r] > m4.x + kRescaleLog2) | (s[r + 1] > m4.y + kRescaleLog2) |
                        (s[r + 2] > m4.z + kRescaleLog2) | (s[r + 3] > m4.w + kRescaleLog2);
              }
            }
          }
        });
      }
      // one vote per tile; a warp that gave up votes too and is caught by the second vote below
      const bool rescale = named_bar_any(bar_id, 128, need || !alive);
      if (rescale) {
        if (named_bar_any(bar_id, 128, !alive)) break;
        with_rows<NP>(nr, [&](auto nr_c) {
          constexpr int HR = group_rows<NP, decltype(nr_c)::value>();
          if constexpr (C::kSpec) {
            if (!first) load_scores(std::integral_constant<int, HR>{});   // s holds this tile's first weights
          }
          warp_columns<HR, true>(s, red + (buf * 4 + wq) * NP + rb, lane);
        });
        named_bar_sync(bar_id, 128);
        // row owners: the maximum moves only for rows whose tile maximum passed it by more than the threshold
        if (ct < hr) {
          const int row = rb + ct;
          float mn = 0.f, neg = -128.f, alpha = 1.f;   // rows past R: no weight
          if (row < R) {
            const float* rr = red + buf * 4 * NP;
            const float tm = fmaxf(fmaxf(rr[row], rr[NP + row]), fmaxf(rr[2 * NP + row], rr[3 * NP + row])) *
                             (C::kSpec ? p.scale_log2 : 1.f);   // (kSpec maxima are of unscaled scores)
            const float mo = first ? kNegInf : m_s[row];
            mn = (first || tm > mo + kRescaleLog2) ? fmaxf(mo, tm) : mo;
            neg = mn == kNegInf ? 0.f : -mn;   // a row that has seen no key yet: masked scores give 2^-inf = 0
            alpha = (mo == kNegInf || mn == mo) ? 1.f : fast_exp2(mo - mn);
          }
          m_s[row] = mn;
          if constexpr (C::kSpec) negm_s[row] = neg;
          alpha_s[buf * NP + row] = alpha;
        }
        named_bar_sync(bar_id, 128);
      }
      with_rows<NP>(nr, [&](auto nr_c) {
        constexpr int HR = group_rows<NP, decltype(nr_c)::value>();
        if constexpr (C::kSpec) {
          if (rescale) {
            // weights against the new maxima; the running sums scale by alpha
            weights(std::integral_constant<int, HR>{});
            const float* al = alpha_s + buf * NP + rb;
#pragma unroll
            for (int r = 0; r < HR; r += 4) {
              const float4 a4 = *reinterpret_cast<const float4*>(al + r);
              const float2 l0 =
                  ffma2(make_float2(l[r], l[r + 1]), make_float2(a4.x, a4.y), make_float2(s[r], s[r + 1]));
              const float2 l1 =
                  ffma2(make_float2(l[r + 2], l[r + 3]), make_float2(a4.z, a4.w), make_float2(s[r + 2], s[r + 3]));
              l[r] = l0.x;
              l[r + 1] = l0.y;
              l[r + 2] = l1.x;
              l[r + 3] = l1.y;
            }
          } else {
#pragma unroll
            for (int r = 0; r < HR; r += 2) {
              const float2 l0 = fadd2(make_float2(l[r], l[r + 1]), make_float2(s[r], s[r + 1]));
              l[r] = l0.x;
              l[r + 1] = l0.y;
            }
          }
          // S(jj) is no longer read: its buffer may take S(jj + 2)
          tc_fence_before();
          mbar_arrive(&bars[B_SEMPTY + buf]);
        } else {
          const float* ms = m_s + rb;
          const float* al = alpha_s + buf * NP + rb;
#pragma unroll
          for (int r = 0; r < HR; r += 4) {
            const float4 m4 = *reinterpret_cast<const float4*>(ms + r);
            const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
            float av[4] = {1.f, 1.f, 1.f, 1.f};
            if (rescale) {
              const float4 a4 = *reinterpret_cast<const float4*>(al + r);
              av[0] = a4.x;
              av[1] = a4.y;
              av[2] = a4.z;
              av[3] = a4.w;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float pr = (s[r + i] == kNegInf) ? 0.f : fast_exp2(s[r + i] - mv[i]);
              l[r + i] = l[r + i] * av[i] + pr;
              s[r + i] = pr;
            }
          }
        }
        // ---- fold the previous tile's O
        auto fold_prev = [&]() {
          if (!first && alive) {
            alive = mbar_wait_warp(&bars[ofull_bar(pbuf(jj - 1))], pphase(jj - 1), abort);
            if (alive) {
              tc_fence_after();
              const float* ap = alpha_s + (buf ^ 1) * NP + rb;
              float ot[HR];
              tmem_ld_cols<HR>(t_lane + (2 + pbuf(jj - 1)) * NP + rb, ot);
              if (rescaled_prev) {
#pragma unroll
                for (int i = 0; i < HR; ++i) o[i] = o[i] * ap[i] + ot[i];
              } else {
#pragma unroll
                for (int i = 0; i < HR; ++i) o[i] += ot[i];
              }
              tc_fence_before();
            }
          }
        };
        if constexpr (C::kPBuf == 1) fold_prev();   // one P buffer: PV(jj-1) must finish before P is rewritten
        if constexpr (C::kOAcc) {
          // P(jj) goes into the buffer PV(jj-2) read.  A tile that moved some row maxima first scales the group's O
          // rows by alpha, once PV(jj-1) has added onto them; PV(jj) then adds this tile's P on top.
          if (rescale && !first && alive) {
            alive = mbar_wait_warp(&bars[ofull_bar(pbuf(jj - 1))], pphase(jj - 1), abort);
            if (alive) {
              tc_fence_after();
              const float* ap = alpha_s + buf * NP + rb;
#pragma unroll
              for (int c = 0; c < HR; c += 8) {   // eight columns at a time: few registers next to P and l
                float ot[8];
                tmem_ld8(t_lane + (2 + ob) * NP + rb + c, ot);
#pragma unroll
                for (int i = 0; i < 8; ++i) ot[i] *= ap[c + i];
                tmem_st8(t_lane + (2 + ob) * NP + rb + c, ot);
              }
              tc_fence_before();
            }
          }
          if (jj >= 2 && alive) alive = mbar_wait_warp(&bars[ofull_bar(pbuf(jj))], pphase(jj - 2), abort);
        }
        // ---- rows past the sequence end may hold stale or uninitialised values: zero V there so P = 0 cannot
        // meet a NaN in the PV product (last tile of a sequence; group 0, before its P arrival)
        if (alive && wg == 0 && L - tok0 < kTileTokens) {
          alive = mbar_wait_warp(&bars[B_VFULL + st], (jj / C::kVStages) & 1, abort);
          if (alive && tok >= L) {
            uint8_t* vrow = smem + C::kV + st * kTileBytes + ct * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0u, 0u, 0u, 0u);
              *reinterpret_cast<uint4*>(vrow + kSlab + c * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
          }
        }
        // ---- P^T (bf16) into its buffer, MN-major without swizzle: 8 consecutive rows of token ct form one 16-byte
        // vector.  Rows past NR (up to the UMMA N) are never read back: their O^T columns are ignored.  The buffer's
        // last reader has finished: PV(jj-1) was folded just above with one buffer; with two, PV(jj-2) was waited for
        // above (O in TMEM) or folded at tile jj-1 or at the end of its segment.
        if (alive) {
          uint8_t* pb = p_smem + pbuf(jj) * NP * 256 + ct * 16 + (rb >> 3) * 2048;
#pragma unroll
          for (int m = 0; m < HR / 8; ++m) {
            uint4 v;
            v.x = pack_bf16x2(s[8 * m + 0], s[8 * m + 1]);
            v.y = pack_bf16x2(s[8 * m + 2], s[8 * m + 3]);
            v.z = pack_bf16x2(s[8 * m + 4], s[8 * m + 5]);
            v.w = pack_bf16x2(s[8 * m + 6], s[8 * m + 7]);
            *reinterpret_cast<uint4*>(pb + m * 2048) = v;
          }
          fence_proxy_async_smem();
          mbar_arrive(&bars[pfull_bar(pbuf(jj))]);
        }
        // two P buffers, O in registers: the fold waits for PV(jj-1) after this tile's P is handed off
        if constexpr (C::kPBuf == 2 && !C::kOAcc) fold_prev();
        if (last && alive) {
          alive = mbar_wait_warp(&bars[ofull_bar(pbuf(jj))], pphase(jj), abort);
          if (alive) {
            tc_fence_after();
            if constexpr (C::kOAcc) {
              tmem_ld_cols<HR>(t_lane + (2 + ob) * NP + rb, o);   // the segment's accumulated O
            } else {
              const float* ap = alpha_s + buf * NP + rb;
              float ot[HR];
              tmem_ld_cols<HR>(t_lane + (2 + pbuf(jj)) * NP + rb, ot);
              if (rescale) {
#pragma unroll
                for (int i = 0; i < HR; ++i) o[i] = o[i] * ap[i] + ot[i];
              } else {
#pragma unroll
                for (int i = 0; i < HR; ++i) o[i] += ot[i];
              }
            }
            tc_fence_before();
            warp_columns<HR, false>(l, lred + wq * NP + rb, lane);
          }
        }
      });
      rescaled_prev = rescale;
      if (named_bar_any(bar_id, 128, !alive)) break;
      if (last) {
        const int c0 = split.owner(seg_b, seg_g, 0), c1 = split.owner(seg_b, seg_g, seg_s1 - seg_s0 - 1);
        const bool complete = c0 == c1;
        const int slot = 2 * blockIdx.x + (seg_s0 < t_begin ? 0 : 1);
        // row owners: 1 / sum, the log2-sum-exp of a piece, and where the row goes
        if (ct < hr) {
          const int r = rb + ct;
          if (r < R) {
            const float lt = lred[r] + lred[NP + r] + lred[2 * NP + r] + lred[3 * NP + r];
            row_inv[r] = lt > 0.f ? 1.f / lt : 0.f;
            if (complete) {
              const int qi = r / G, h = r - qi * G;
              row_out[r] = (int64_t)(q0 + qi) * p.out_row_stride + (int64_t)(seg_g * G + h) * kHeadDim;
            } else {
              row_out[r] = ((int64_t)slot * NP + r) * kHeadDim;
              p.part_lse[slot * NP + r] = lt > 0.f ? m_s[r] + __log2f(lt) : kNegInf;
            }
          }
        }
        named_bar_sync(bar_id, 128);
        with_rows<NP>(nr, [&](auto nr_c) {
          constexpr int HR = group_rows<NP, decltype(nr_c)::value>();
#pragma unroll
          for (int i = 0; i < HR; ++i) {
            const int r = rb + i;
            if (r < R) {
              const float val = o[i] * row_inv[r];
              if (complete) {
                p.out[row_out[r] + ct] = __float2bfloat16_rn(val);
              } else {
                p.part_o[row_out[r] + ct] = val;
              }
            }
          }
        });
        if (!complete) arrive_and_merge(c0, c1, rb, hr);
      }
    }
  }

  named_bar_sync(3, C::kThreads - 64);
  if (*abort) {
    // a wait gave up: let any copy or MMA still in flight land before the shared memory and TMEM go away
    if (tid == kConsumerBase) atomicOr(&g_error_word, kErrTimeout);
    for (int i = 0; i < 1000; ++i) sleep_ns(1000);
    named_bar_sync(3, C::kThreads - 64);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

template <int NP, bool Spec = false>
cudaError_t launch_np(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const DecodeParams& p, int grid,
                      cudaStream_t stream, bool pdl) {
  constexpr int smem = Cfg<NP, Spec>::kBytes;
  static_assert(smem <= 232448, "shared memory budget");
  cudaError_t e =
      cudaFuncSetAttribute(paged_decode_kernel<NP, Spec>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return launch_kernel(paged_decode_kernel<NP, Spec>, dim3(grid), dim3(Cfg<NP, Spec>::kThreads), smem, stream, pdl,
                       tm_k, tm_v, p);
}

}  // namespace

int decode_rows_padded(int rows) {
  // 9-16 rows take the 32-row instantiation, whose two softmax groups split them 8 + 8 (the 16-row one has a
  // single group)
  if (rows <= 8) return 16;
  if (rows <= 32) return 32;
  if (rows <= 48) return 48;
  return 0;
}

// Workspace: the merge tickets first, at the same place for every row width and call kind (a workspace shared by
// several kinds of call keeps them zero between calls), then the partials.
static size_t ticket_bytes(int grid) {
  return (kTicketStride * static_cast<size_t>(grid) * sizeof(int32_t) + 255) & ~size_t(255);
}

size_t decode_workspace_bytes(int grid, int np) {
  return ticket_bytes(grid) + static_cast<size_t>(2) * grid * np * (kHeadDim + 1) * sizeof(float);
}

void decode_workspace_layout(void* ws, int grid, int np, DecodeParams* p) {
  p->counters = static_cast<int32_t*>(ws);
  p->part_o = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + ticket_bytes(grid));
  p->part_lse = p->part_o + static_cast<size_t>(2) * grid * np * kHeadDim;
}

cudaError_t launch_paged_decode(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const DecodeParams& params,
                                int np, int grid, cudaStream_t stream, bool pdl) {
  DecodeParams p = params;
  p.pdl = pdl ? 1 : 0;
  switch (np) {
    case 16: return launch_np<16>(tm_k, tm_v, p, grid, stream, pdl);
    case 32: return launch_np<32>(tm_k, tm_v, p, grid, stream, pdl);
    // fixed-length batches of 33-48 rows (verify with many drafts) take the speculative-weights variant; varlen
    // calls, whose short runs are mostly 1-row decode segments, the plain one
    case 48: return p.cu_q == nullptr ? launch_np<48, true>(tm_k, tm_v, p, grid, stream, pdl)
                                      : launch_np<48>(tm_k, tm_v, p, grid, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nva
