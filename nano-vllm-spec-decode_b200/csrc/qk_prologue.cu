// The attention prologue of Qwen3 in one pass (nanovllm/models/qwen3.py:88-97 followed by the KV scatter of
// Attention.forward, nanovllm/layers/attention.py:61-62): from the fused q/k/v projection output,
//   q_out = rope(rmsnorm(q) * q_norm_w),  k' = rope(rmsnorm(k) * k_norm_w),
//   k_cache[slot] = k', v_cache[slot] = v   (slot = slot_mapping[token], skipped when -1),  optionally k_out = k'.
// RMSNorm (layers/layernorm.py:16-26) over each head's 128 dims in float32 with the reference's rounding points:
// x * rsqrt(mean(x^2) + eps) rounded to bf16, then times the bf16 weight, rounded to bf16.  Rotary
// (layers/rotary_embedding.py:6-14, 37-48): rotate-half on the float32 values with the reference's float32
// cos / sin table (cos in the first 64 columns of a position's row, sin in the last 64), rounded to bf16.
//
// One block per token and one warp per group of 8 of its heads -- heads ordered q, then k, then v -- with 4 dims per
// lane: the warp issues the 8-byte loads of all its heads first, reads the token's cos / sin values and the norm
// weights once, then normalises, rotates and stores head by head (the rotate-half partner of lane l's dims is lane
// l ^ 16), in packed f32x2 arithmetic.  Each element is read once and written once or twice; no shared memory.
#include "nva_ptx.cuh"
#include "nva_kernels.h"

namespace nva {

namespace {

constexpr int kHeadsPerWarp = 8;   // heads of one token per warp: their loads in flight together, one cos/sin read

// Rounds a pair to bf16 (round to nearest even, one packed conversion) and widens it back to float32.
__device__ __forceinline__ float2 bf16r2(float2 v) {
  const __nv_bfloat162 b = __float22bfloat162_rn(v);
  return __bfloat1622float2(b);
}

// One block per token, one warp per group of 8 heads (q heads, then k heads, then v heads).
__global__ void __launch_bounds__(256, 4)
qk_prologue_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t qkv_stride, int32_t H, int32_t KVH,
                   const int64_t* __restrict__ positions, const float* __restrict__ cos_sin, int32_t max_pos,
                   const __nv_bfloat16* __restrict__ q_w, const __nv_bfloat16* __restrict__ k_w, float eps,
                   __nv_bfloat16* __restrict__ q_out, int64_t q_out_stride, __nv_bfloat16* __restrict__ k_out,
                   int64_t k_out_stride, __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                   int64_t num_slots, const int32_t* __restrict__ slots) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x;
  const int heads = H + 2 * KVH;
  const int h0 = (threadIdx.x >> 5) * kHeadsPerWarp;
  const int nh = min(kHeadsPerWarp, heads - h0);
  // every load of the warp first: its heads' rows, the token's slot, position and cos / sin values, the weights
  const __nv_bfloat16* src = qkv + t * qkv_stride + h0 * kHeadDim + lane * 4;
  uint2 raw[kHeadsPerWarp];
#pragma unroll
  for (int i = 0; i < kHeadsPerWarp; ++i)
    if (i < nh) raw[i] = *reinterpret_cast<const uint2*>(src + i * kHeadDim);
  const bool has_kv = h0 + nh > H;
  const int32_t slot = (has_kv && slots != nullptr) ? __ldg(slots + t) : -1;
  const bool store = slot >= 0 && slot < num_slots;
  if (has_kv && slots != nullptr && slot >= num_slots && lane == 0 && h0 <= H) atomicOr(&g_error_word, kErrSlotRange);
  float2 c01 = make_float2(0.f, 0.f), c23 = c01, s01 = c01, s23 = c01, qw01 = c01, qw23 = c01, kw01 = c01, kw23 = c01;
  if (h0 < H + KVH) {
    int64_t pos = __ldg(positions + t);
    pos = pos < 0 ? 0 : (pos >= max_pos ? max_pos - 1 : pos);
    const int c = (lane & 15) * 4;
    const float4 cs = *reinterpret_cast<const float4*>(cos_sin + pos * kHeadDim + c);
    const float4 sn = *reinterpret_cast<const float4*>(cos_sin + pos * kHeadDim + 64 + c);
    // x1' = x1 c - x2 s (dims < 64), x2' = x2 c + x1 s: the partner's term enters with sin negated below dim 64
    const float sg = lane < 16 ? -1.f : 1.f;
    c01 = make_float2(cs.x, cs.y);
    c23 = make_float2(cs.z, cs.w);
    s01 = make_float2(sg * sn.x, sg * sn.y);
    s23 = make_float2(sg * sn.z, sg * sn.w);
    const uint2 qwr = *reinterpret_cast<const uint2*>(q_w + lane * 4);
    const uint2 kwr = *reinterpret_cast<const uint2*>(k_w + lane * 4);
    qw01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qwr.x));
    qw23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qwr.y));
    kw01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kwr.x));
    kw23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kwr.y));
  }
  const int64_t row_elems = static_cast<int64_t>(KVH) * kHeadDim;
#pragma unroll
  for (int i = 0; i < kHeadsPerWarp; ++i) {
    const int h = h0 + i;
    if (i >= nh) break;
    if (h >= H + KVH) {   // value head: copied into the cache as is
      if (store) *reinterpret_cast<uint2*>(v_cache + slot * row_elems + (h - H - KVH) * kHeadDim + lane * 4) = raw[i];
      continue;
    }
    float2 x01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[i].x));
    float2 x23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw[i].y));
    float ss = x01.x * x01.x + x01.y * x01.y + x23.x * x23.x + x23.y * x23.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss * (1.0f / kHeadDim) + eps);
    const bool is_q = h < H;
    // RMSNorm with the reference's rounding points: x * inv to bf16, times the bf16 weight, to bf16
    const float2 iv = make_float2(inv, inv);
    x01 = bf16r2(fmul2(bf16r2(fmul2(x01, iv)), is_q ? qw01 : kw01));
    x23 = bf16r2(fmul2(bf16r2(fmul2(x23, iv)), is_q ? qw23 : kw23));
    // rotate-half: dims d < 64 pair with d + 64 (lane l with lane l ^ 16); each product rounded on its own, as
    // torch's elementwise float32 ops do (no fused multiply-add)
    const float2 y01 = make_float2(__shfl_xor_sync(0xffffffffu, x01.x, 16), __shfl_xor_sync(0xffffffffu, x01.y, 16));
    const float2 y23 = make_float2(__shfl_xor_sync(0xffffffffu, x23.x, 16), __shfl_xor_sync(0xffffffffu, x23.y, 16));
    const float2 r01 = fadd2(fmul2(x01, c01), fmul2(y01, s01));
    const float2 r23 = fadd2(fmul2(x23, c23), fmul2(y23, s23));
    uint2 packed;
    packed.x = pack_bf16x2(r01.x, r01.y);
    packed.y = pack_bf16x2(r23.x, r23.y);
    if (is_q) {
      *reinterpret_cast<uint2*>(q_out + t * q_out_stride + h * kHeadDim + lane * 4) = packed;
      continue;
    }
    const int kh = h - H;
    if (k_out != nullptr) *reinterpret_cast<uint2*>(k_out + t * k_out_stride + kh * kHeadDim + lane * 4) = packed;
    if (store) *reinterpret_cast<uint2*>(k_cache + slot * row_elems + kh * kHeadDim + lane * 4) = packed;
  }
}

}  // namespace

cudaError_t launch_qk_prologue(const void* qkv, int64_t qkv_stride, int32_t T, int32_t H, int32_t KVH,
                               const int64_t* positions, const float* cos_sin, int32_t max_pos, const void* q_w,
                               const void* k_w, float eps, void* q_out, int64_t q_out_stride, void* k_out,
                               int64_t k_out_stride, void* k_cache, void* v_cache, int64_t num_slots,
                               const int32_t* slots, cudaStream_t stream) {
  const int groups = (H + 2 * KVH + kHeadsPerWarp - 1) / kHeadsPerWarp;
  if (groups > 8) return cudaErrorInvalidValue;   // one block of at most 256 threads per token
  qk_prologue_kernel<<<static_cast<unsigned>(T), 32 * groups, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(qkv), qkv_stride, H, KVH, positions, cos_sin, max_pos,
      static_cast<const __nv_bfloat16*>(q_w), static_cast<const __nv_bfloat16*>(k_w), eps,
      static_cast<__nv_bfloat16*>(q_out), q_out_stride, static_cast<__nv_bfloat16*>(k_out), k_out_stride,
      static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), num_slots, slots);
  return cudaGetLastError();
}

}  // namespace nva
