// The attention prologue of Qwen3 in one pass (nanovllm/models/qwen3.py:88-97 followed by the KV scatter of
// Attention.forward, nanovllm/layers/attention.py:61-62): from the fused q/k/v projection output,
//   q_out = rope(rmsnorm(q) * q_norm_w),  k' = rope(rmsnorm(k) * k_norm_w),
//   k_cache[slot] = k', v_cache[slot] = v   (slot = slot_mapping[token], skipped when -1),  optionally k_out = k'.
// RMSNorm (layers/layernorm.py:16-26) over each head's 128 dims in float32 with the reference's rounding points:
// x * rsqrt(mean(x^2) + eps) rounded to bf16, then times the bf16 weight, rounded to bf16.  Rotary
// (layers/rotary_embedding.py:6-14, 37-48): rotate-half on the float32 values with the reference's float32
// cos / sin table (cos in the first 64 columns of a position's row, sin in the last 64), rounded to bf16.
//
// One warp per (token, head) -- q heads, then k heads, then v heads -- and 4 dims per lane (8-byte loads); the
// rotate-half partner of lane l's dims is lane l ^ 16.  HBM / latency bound: each element is read once and written
// once or twice; no shared memory.
#include "nva_ptx.cuh"
#include "nva_kernels.h"

namespace nva {

namespace {

constexpr int kProThreads = 256;

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(kProThreads)
qk_prologue_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t qkv_stride, int32_t T, int32_t H, int32_t KVH,
                   const int64_t* __restrict__ positions, const float* __restrict__ cos_sin, int32_t max_pos,
                   const __nv_bfloat16* __restrict__ q_w, const __nv_bfloat16* __restrict__ k_w, float eps,
                   __nv_bfloat16* __restrict__ q_out, int64_t q_out_stride, __nv_bfloat16* __restrict__ k_out,
                   int64_t k_out_stride, __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                   int64_t num_slots, const int32_t* __restrict__ slots) {
  const int lane = threadIdx.x & 31;
  const int64_t unit = (static_cast<int64_t>(blockIdx.x) * kProThreads + threadIdx.x) >> 5;
  const int heads = H + 2 * KVH;
  if (unit >= static_cast<int64_t>(T) * heads) return;
  const int t = static_cast<int>(unit / heads);
  const int h = static_cast<int>(unit - static_cast<int64_t>(t) * heads);
  const __nv_bfloat16* src = qkv + t * qkv_stride + h * kHeadDim + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  const int32_t slot = (h >= H && slots != nullptr) ? __ldg(slots + t) : -1;
  const bool store = slot >= 0 && slot < num_slots;
  if (h >= H && slots != nullptr && slot >= num_slots) {
    if (lane == 0 && h == H) atomicOr(&g_error_word, kErrSlotRange);
  }
  const int64_t row_elems = static_cast<int64_t>(KVH) * kHeadDim;
  if (h >= H + KVH) {   // value head: copied into the cache as is
    if (store)
      *reinterpret_cast<uint2*>(v_cache + slot * row_elems + (h - H - KVH) * kHeadDim + lane * 4) = raw;
    return;
  }
  float x[4];
  {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    x[0] = __low2float(a);
    x[1] = __high2float(a);
    x[2] = __low2float(b);
    x[3] = __high2float(b);
  }
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss * (1.0f / kHeadDim) + eps);
  const bool is_q = h < H;
  const __nv_bfloat16* w = (is_q ? q_w : k_w) + lane * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = bf16r(__fmul_rn(bf16r(__fmul_rn(x[i], inv)), __bfloat162float(w[i])));
  // rotate-half: dims d < 64 pair with d + 64 (lane l with lane l ^ 16)
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) y[i] = __shfl_xor_sync(0xffffffffu, x[i], 16);
  int64_t pos = __ldg(positions + t);
  pos = pos < 0 ? 0 : (pos >= max_pos ? max_pos - 1 : pos);
  const int c = (lane & 15) * 4;
  const float4 cs = *reinterpret_cast<const float4*>(cos_sin + pos * kHeadDim + c);
  const float4 sn = *reinterpret_cast<const float4*>(cos_sin + pos * kHeadDim + 64 + c);
  const float cv[4] = {cs.x, cs.y, cs.z, cs.w}, sv[4] = {sn.x, sn.y, sn.z, sn.w};
  float r[4];
  // each product rounded on its own, as torch's elementwise float32 ops do (no fused multiply-add)
  if (lane < 16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = __fsub_rn(__fmul_rn(x[i], cv[i]), __fmul_rn(y[i], sv[i]));   // x1 cos - x2 sin
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = __fadd_rn(__fmul_rn(x[i], cv[i]), __fmul_rn(y[i], sv[i]));   // x2 cos + x1 sin
  }
  uint2 packed;
  packed.x = pack_bf16x2(r[0], r[1]);
  packed.y = pack_bf16x2(r[2], r[3]);
  if (is_q) {
    *reinterpret_cast<uint2*>(q_out + t * q_out_stride + h * kHeadDim + lane * 4) = packed;
    return;
  }
  const int kh = h - H;
  if (k_out != nullptr) *reinterpret_cast<uint2*>(k_out + t * k_out_stride + kh * kHeadDim + lane * 4) = packed;
  if (store) *reinterpret_cast<uint2*>(k_cache + slot * row_elems + kh * kHeadDim + lane * 4) = packed;
}

}  // namespace

cudaError_t launch_qk_prologue(const void* qkv, int64_t qkv_stride, int32_t T, int32_t H, int32_t KVH,
                               const int64_t* positions, const float* cos_sin, int32_t max_pos, const void* q_w,
                               const void* k_w, float eps, void* q_out, int64_t q_out_stride, void* k_out,
                               int64_t k_out_stride, void* k_cache, void* v_cache, int64_t num_slots,
                               const int32_t* slots, cudaStream_t stream) {
  const int64_t warps = static_cast<int64_t>(T) * (H + 2 * KVH);
  const int64_t blocks = (warps * 32 + kProThreads - 1) / kProThreads;
  qk_prologue_kernel<<<static_cast<unsigned>(blocks), kProThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(qkv), qkv_stride, T, H, KVH, positions, cos_sin, max_pos,
      static_cast<const __nv_bfloat16*>(q_w), static_cast<const __nv_bfloat16*>(k_w), eps,
      static_cast<__nv_bfloat16*>(q_out), q_out_stride, static_cast<__nv_bfloat16*>(k_out), k_out_stride,
      static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), num_slots, slots);
  return cudaGetLastError();
}

}  // namespace nva
