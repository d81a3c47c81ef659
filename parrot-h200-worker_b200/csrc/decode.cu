// Single-token decode attention with the position in device memory, so that
// a whole decode step can be captured once and replayed.
//
// One query token per batch row attends over the cached keys [lo, pos] of its
// KV head (lo = max(0, pos - window + 1)) after its own key/value are appended
// at pos.  Two layouts share the kernels:
//   local GQA (model.py:303-328): q [B, H, D] bf16, separate K and V caches
//                [B, KVH, S, D], G = H / KVH query heads per KV head;
//   MLA absorbed (model.py:399-432): q [B, H, L] fp32 (the absorbed query),
//                one latent cache [B, S, L] serving as both K and V for all H
//                heads (KVH = 1, G = H).
// Split over the keys (flash-decoding): CTA (chunk, kv head, batch row) takes
// 128 keys, one warp per query head of the group; it stages the chunk's keys
// and values in shared memory, computes fp32 scores, a chunk-local softmax and
// the weighted value sum, and writes (max, sum, acc[D]) partials.  A merge
// kernel (one warp per (batch row, head)) rescales and adds the chunks in
// order, so the result does not depend on timing.  The CTA whose chunk holds
// pos also writes the new key/value into the cache (no other CTA reads that
// row).  The position is read from device memory and checked against the
// cache length; a bad position is reported in the status word and the CTA
// writes nothing.
#include "common.cuh"
#include "kernels.h"

namespace parrot {

constexpr int kDecodeChunk = 128;  // keys per CTA

template <int D, int G>
__global__ void __launch_bounds__(32 * G) decode_attn_partial_kernel(DecodeAttnArgs a) {
  constexpr int NV = D / 8;  // 16-byte vectors per row
  extern __shared__ __align__(16) unsigned char dec_smem[];
  uint4* k_s = reinterpret_cast<uint4*>(dec_smem);            // [chunk][NV]
  uint4* v_s = k_s + kDecodeChunk * NV;                       // [chunk][NV] (unused: V = K)
  float* q_s = reinterpret_cast<float*>(v_s + (a.v_cache != nullptr ? kDecodeChunk * NV : 0));
  float* p_s = q_s + G * D;                                   // [G][chunk]

  const int chunk = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = kvh * G + warp;  // this warp's query head
  griddep_wait();
  griddep_launch();
  const int pos = __ldg(a.pos);
  float* part = a.part + (((size_t)b * a.H + h) * a.n_chunks + chunk) * (D + 2);
  if (pos < 0 || pos >= a.S) {
    if (threadIdx.x == 0) report_status(a.status, kStatusBadIndex, 40, pos);
    return;
  }
  const int lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  const int k0 = max(lo, chunk * kDecodeChunk), k1 = min(pos + 1, (chunk + 1) * kDecodeChunk);
  if (k0 >= k1) {  // no key of this chunk is visible: an empty partial
    if (lane == 0) {
      part[D] = -INFINITY;
      part[D + 1] = 0.f;
    }
    return;
  }
  const int n = k1 - k0;
  const size_t row0 = ((size_t)b * a.KVH + kvh) * a.S;
  const uint4* kc = reinterpret_cast<const uint4*>(a.k_cache + row0 * D);
  const uint4* vc = a.v_cache != nullptr ? reinterpret_cast<const uint4*>(a.v_cache + row0 * D)
                                         : nullptr;
  const uint4* kn = reinterpret_cast<const uint4*>(a.k_new + (size_t)b * a.kv_row + (size_t)kvh * D);
  const uint4* vn =
      a.v_new != nullptr
          ? reinterpret_cast<const uint4*>(a.v_new + (size_t)b * a.kv_row + (size_t)kvh * D)
          : nullptr;
  // stage the chunk's keys (and values); the row at pos comes from the new token
  for (int i = threadIdx.x; i < n * NV; i += blockDim.x) {
    const int j = i / NV, c = i - j * NV;
    const int key = k0 + j;
    if (key == pos) {
      k_s[i] = __ldg(kn + c);
      if (vc != nullptr) v_s[i] = __ldg(vn + c);
    } else {
      cp_async16(k_s + i, kc + (size_t)key * NV + c);
      if (vc != nullptr) cp_async16(v_s + i, vc + (size_t)key * NV + c);
    }
  }
  // this warp's query, as fp32
  for (int d = lane; d < D; d += 32) {
    const size_t qi = (size_t)b * a.q_row + (size_t)h * D + d;
    const float qv = a.q_f32 ? __ldg(static_cast<const float*>(a.q) + qi)
                             : __bfloat162float(static_cast<const __nv_bfloat16*>(a.q)[qi]);
    q_s[warp * D + d] = qv;
  }
  cp_async_wait_all();
  __syncthreads();
  if (pos >= k0 && pos < k1 && warp == 0) {
    // append the new token to the cache (only this CTA touches row pos)
    uint4* kw = reinterpret_cast<uint4*>(a.k_cache + (row0 + pos) * D);
    uint4* vw = a.v_cache != nullptr ? reinterpret_cast<uint4*>(a.v_cache + (row0 + pos) * D)
                                     : nullptr;
    for (int c = lane; c < NV; c += 32) {
      kw[c] = k_s[(pos - k0) * NV + c];
      if (vw != nullptr) vw[c] = v_s[(pos - k0) * NV + c];
    }
  }

  // scores: lane l takes keys l, l + 32, ...
  const float* q = q_s + warp * D;
  float m = -INFINITY;
  for (int j = lane; j < n; j += 32) {
    const uint4* kr = k_s + j * NV;
    float s = 0.f;
#pragma unroll 4
    for (int c = 0; c < NV; ++c) {
      float f[8];
      bf16x8_to_float(kr[c], f);
#pragma unroll
      for (int t = 0; t < 8; ++t) s = fmaf(q[c * 8 + t], f[t], s);
    }
    s *= a.scale;
    p_s[warp * kDecodeChunk + j] = s;
    m = fmaxf(m, s);
  }
  m = warp_max(m);
  float l = 0.f;
  for (int j = lane; j < n; j += 32) {
    const float e = __expf(p_s[warp * kDecodeChunk + j] - m);
    p_s[warp * kDecodeChunk + j] = e;
    l += e;
  }
  l = warp_sum(l);
  __syncwarp();
  // weighted values: lane l owns dims l, l + 32, ...
  const uint4* vsrc = vc != nullptr ? v_s : k_s;
  const __nv_bfloat16* vrow = reinterpret_cast<const __nv_bfloat16*>(vsrc);
  for (int d = lane; d < D; d += 32) {
    float acc = 0.f;
    for (int j = 0; j < n; ++j)
      acc = fmaf(p_s[warp * kDecodeChunk + j], __bfloat162float(vrow[(size_t)j * D + d]), acc);
    part[d] = acc;
  }
  if (lane == 0) {
    part[D] = m;
    part[D + 1] = l;
  }
}

template <int D>
__global__ void __launch_bounds__(128) decode_attn_merge_kernel(DecodeAttnArgs a) {
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x * 4 + (threadIdx.x >> 5);  // (batch row, head)
  griddep_wait();
  griddep_launch();
  if (bh >= a.B * a.H) return;
  const int pos = __ldg(a.pos);
  if (pos < 0 || pos >= a.S) return;  // reported by the partial kernel
  const int lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  const int c0 = lo / kDecodeChunk, c1 = pos / kDecodeChunk;
  const float* part = a.part + (size_t)bh * a.n_chunks * (D + 2);
  float mx = -INFINITY;
  for (int c = c0; c <= c1; ++c) mx = fmaxf(mx, part[(size_t)c * (D + 2) + D]);
  float acc[(D + 31) / 32] = {};
  float l = 0.f;
  for (int c = c0; c <= c1; ++c) {
    const float* pc = part + (size_t)c * (D + 2);
    const float w = __expf(pc[D] - mx);
    l = fmaf(w, pc[D + 1], l);
#pragma unroll
    for (int i = 0; i < (D + 31) / 32; ++i) {
      const int d = lane + 32 * i;
      if (d < D) acc[i] = fmaf(w, pc[d], acc[i]);
    }
  }
  const float inv = 1.0f / l;
#pragma unroll
  for (int i = 0; i < (D + 31) / 32; ++i) {
    const int d = lane + 32 * i;
    if (d >= D) continue;
    const size_t oi = (size_t)bh * D + d;
    if (a.out_f32)
      static_cast<float*>(a.out)[oi] = acc[i] * inv;
    else
      static_cast<__nv_bfloat16*>(a.out)[oi] = __float2bfloat16_rn(acc[i] * inv);
  }
}

int decode_attn_chunks(int max_positions) {
  return (max_positions + kDecodeChunk - 1) / kDecodeChunk;
}

template <int D, int G>
static int launch_decode_dg(const DecodeAttnArgs& a, cudaStream_t stream) {
  const size_t smem = (size_t)kDecodeChunk * (D / 8) * 16 * (a.v_cache != nullptr ? 2 : 1) +
                      (size_t)G * D * 4 + (size_t)G * kDecodeChunk * 4;
  static unsigned long long configured = 0;  // per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -2;
  if (!(configured & (1ull << dev))) {
    const int max_smem = kDecodeChunk * (D / 8) * 16 * 2 + G * D * 4 + G * kDecodeChunk * 4;
    if (cudaFuncSetAttribute(decode_attn_partial_kernel<D, G>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) != cudaSuccess)
      return -2;
    configured |= 1ull << dev;
  }
  if (launch_pdl(decode_attn_partial_kernel<D, G>, dim3(a.n_chunks, a.KVH, a.B), dim3(32 * G),
                 smem, stream, a) != cudaSuccess)
    return -2;
  return launch_pdl(decode_attn_merge_kernel<D>, dim3((a.B * a.H + 3) / 4), dim3(128), 0, stream,
                    a) == cudaSuccess
             ? 0
             : -2;
}

int launch_decode_attention(const DecodeAttnArgs& a, cudaStream_t stream) {
  if (a.B == 0) return 0;
  const int G = a.H / a.KVH;
  if (a.D == 96 && G == 4) return launch_decode_dg<96, 4>(a, stream);
  if (a.D == 96 && G == 1) return launch_decode_dg<96, 1>(a, stream);
  if (a.D == 128 && G == 8) return launch_decode_dg<128, 8>(a, stream);
  if (a.D == 32 && G == 2) return launch_decode_dg<32, 2>(a, stream);
  if (a.D == 32 && G == 4) return launch_decode_dg<32, 4>(a, stream);
  return -1;
}

}  // namespace parrot
