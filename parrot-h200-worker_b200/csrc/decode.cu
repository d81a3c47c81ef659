// Single-token decode attention with the position in device memory, so that
// a whole decode step can be captured once and replayed.
//
// One query token per batch row attends over the cached keys [lo, pos] of its
// KV head (lo = max(0, pos - window + 1)) after its own key/value are appended
// at pos.  Two layouts share the kernel:
//   local GQA (model.py:303-328): q [B, H, D] bf16, separate K and V caches
//                [B, KVH, S, D], G = H / KVH query heads per KV head;
//   MLA absorbed (model.py:399-432): q [B, H, L] fp32 (the absorbed query),
//                one latent cache [B, S, L] serving as both K and V for all H
//                heads (KVH = 1, G = H).
// Split over the keys (flash-decoding) in one launch: the visible keys are cut
// into 32-key chunks (one key per lane); CTA (slot, kv head, batch row) takes
// chunks slot, slot + slots, ... with one warp per query head of the group,
// stages each chunk's keys and values in shared memory (rows padded to an odd
// number of 16-byte vectors, so the lane-per-key reads are conflict-free) and
// keeps an online softmax (running max, sum and fp32 weighted values).  A
// group whose keys fit one chunk finishes in that CTA; otherwise every CTA
// writes its (max, sum, acc[D]) partial, and the last CTA of the group to
// arrive (an atomic counter that it resets) merges the partials in slot order,
// so the result does not depend on timing.  The CTA whose chunk holds pos also
// writes the new key/value into the cache (no other CTA reads that row).  The
// position is read from device memory and checked against the cache length; a
// bad position is reported in the status word and nothing is written.  With
// RoPE tables given (local GQA), the kernel rotates the query as it loads it
// and the new key as it stages and appends it, so no separate RoPE launch runs.
#include "common.cuh"
#include "kernels.h"

namespace parrot {

constexpr int kDecodeChunk = 32;  // keys per chunk: one per lane

// Rotary embedding of one bf16 pair at table row `pos`, column pair j, with
// the rounding of the RoPE kernel (every product and the sum rounded to bf16).
__device__ __forceinline__ float2 rope_pair(float e, float o, const DecodeAttnArgs& a, int pos,
                                            int j) {
  const size_t t = (size_t)pos * (a.D >> 1) + j;
  const float c = __bfloat162float(a.cos_t[t]), s = __bfloat162float(a.sin_t[t]);
  return make_float2(round_bf16(round_bf16(e * c) - round_bf16(o * s)),
                     round_bf16(round_bf16(e * s) + round_bf16(o * c)));
}

// The key vector cv (columns 8 cv .. 8 cv + 7) of the new token, rotated.
__device__ __forceinline__ uint4 rope_vec8(uint4 v, const DecodeAttnArgs& a, int pos, int cv) {
  float f[8];
  bf16x8_to_float(v, f);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 r = rope_pair(f[2 * k], f[2 * k + 1], a, pos, cv * 4 + k);
    f[2 * k] = r.x;
    f[2 * k + 1] = r.y;
  }
  return float_to_bf16x8(f);
}

template <int D, int G>
__global__ void __launch_bounds__(32 * G) decode_attn_kernel(DecodeAttnArgs a) {
  constexpr int NV = D / 8;             // 16-byte vectors per row
  constexpr int NVP = NV | 1;           // staged row stride in vectors (odd)
  constexpr int NP = D / 2;             // bf16 pairs per row
  constexpr int PPL = (NP + 31) / 32;   // pairs per lane
  extern __shared__ __align__(16) unsigned char dec_smem[];
  __shared__ int last_s;
  const bool sep_v = a.v_cache != nullptr;
  uint4* k_s = reinterpret_cast<uint4*>(dec_smem);  // [chunk][NVP]
  uint4* v_s = sep_v ? k_s + kDecodeChunk * NVP : k_s;
  float* q_s = reinterpret_cast<float*>(k_s + kDecodeChunk * NVP * (sep_v ? 2 : 1));  // [G][D]
  float* p_s = q_s + G * D;                                                           // [G][chunk]

  const int slot = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = kvh * G + warp;  // this warp's query head
  griddep_wait();
  griddep_launch();
  const int pos = __ldg(a.pos);
  if (pos < 0 || pos >= a.S) {
    if (threadIdx.x == 0) report_status(a.status, kStatusBadIndex, 40, pos);
    return;
  }
  const int lo = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  const int c_first = lo / kDecodeChunk, c_last = pos / kDecodeChunk;
  const int busy = min(a.slots, c_last - c_first + 1);  // CTAs of this group with keys
  if (slot >= busy) return;
  const size_t row0 = ((size_t)b * a.KVH + kvh) * a.S;
  const uint4* kc = reinterpret_cast<const uint4*>(a.k_cache + row0 * D);
  const uint4* vc = sep_v ? reinterpret_cast<const uint4*>(a.v_cache + row0 * D) : nullptr;
  const uint4* kn = reinterpret_cast<const uint4*>(a.k_new + (size_t)b * a.kv_row + (size_t)kvh * D);
  const uint4* vn =
      sep_v ? reinterpret_cast<const uint4*>(a.v_new + (size_t)b * a.kv_row + (size_t)kvh * D)
            : nullptr;
  // this warp's query, as fp32 (rotated here when the tables are given)
  if (a.cos_t != nullptr) {
    const __nv_bfloat162* qp = reinterpret_cast<const __nv_bfloat162*>(
        static_cast<const __nv_bfloat16*>(a.q) + (size_t)b * a.q_row + (size_t)h * D);
    for (int j = lane; j < D / 2; j += 32) {
      const float2 e = __bfloat1622float2(qp[j]);
      const float2 r = rope_pair(e.x, e.y, a, pos, j);
      q_s[warp * D + 2 * j] = r.x;
      q_s[warp * D + 2 * j + 1] = r.y;
    }
  } else {
    for (int d = lane; d < D; d += 32) {
      const size_t qi = (size_t)b * a.q_row + (size_t)h * D + d;
      q_s[warp * D + d] = a.q_f32 ? __ldg(static_cast<const float*>(a.q) + qi)
                                  : __bfloat162float(static_cast<const __nv_bfloat16*>(a.q)[qi]);
    }
  }

  float m = -INFINITY, l = 0.f;
  float2 acc[PPL];
#pragma unroll
  for (int i = 0; i < PPL; ++i) acc[i] = make_float2(0.f, 0.f);
  const uint32_t* vw32 = reinterpret_cast<const uint32_t*>(v_s);
  for (int c = c_first + slot; c <= c_last; c += a.slots) {
    const int k0 = max(lo, c * kDecodeChunk), k1 = min(pos + 1, (c + 1) * kDecodeChunk);
    const int n = k1 - k0;  // >= 1
    __syncthreads();        // the previous chunk's rows are consumed
    // stage the chunk's keys (and values); the row at pos comes from the new
    // token, which this CTA also appends to the cache
    for (int i = threadIdx.x; i < n * NV; i += blockDim.x) {
      const int j = i / NV, cv = i - j * NV;
      const int key = k0 + j;
      if (key == pos) {
        const uint4 kv = a.cos_t != nullptr ? rope_vec8(__ldg(kn + cv), a, pos, cv) : __ldg(kn + cv);
        k_s[j * NVP + cv] = kv;
        reinterpret_cast<uint4*>(a.k_cache + (row0 + pos) * D)[cv] = kv;
        if (sep_v) {
          const uint4 vv = __ldg(vn + cv);
          v_s[j * NVP + cv] = vv;
          reinterpret_cast<uint4*>(a.v_cache + (row0 + pos) * D)[cv] = vv;
        }
      } else {
        cp_async16(k_s + j * NVP + cv, kc + (size_t)key * NV + cv);
        if (sep_v) cp_async16(v_s + j * NVP + cv, vc + (size_t)key * NV + cv);
      }
    }
    cp_async_wait_all();
    __syncthreads();
    // score of key k0 + lane
    float s = -INFINITY;
    if (lane < n) {
      const uint4* kr = k_s + lane * NVP;
      const float* q = q_s + warp * D;
      float dot = 0.f;
#pragma unroll
      for (int cv = 0; cv < NV; ++cv) {
        float f[8];
        bf16x8_to_float(kr[cv], f);
        const float4 qa = *reinterpret_cast<const float4*>(q + cv * 8);
        const float4 qb = *reinterpret_cast<const float4*>(q + cv * 8 + 4);
        dot = fmaf(qa.x, f[0], dot);
        dot = fmaf(qa.y, f[1], dot);
        dot = fmaf(qa.z, f[2], dot);
        dot = fmaf(qa.w, f[3], dot);
        dot = fmaf(qb.x, f[4], dot);
        dot = fmaf(qb.y, f[5], dot);
        dot = fmaf(qb.z, f[6], dot);
        dot = fmaf(qb.w, f[7], dot);
      }
      s = dot * a.scale;
    }
    // online softmax: lane 0 always holds a key, so the new max is finite
    const float mn = fmaxf(m, warp_max(s));
    const float corr = __expf(m - mn);  // 0 on the first chunk
    const float p = lane < n ? __expf(s - mn) : 0.f;
    l = fmaf(l, corr, warp_sum(p));
    m = mn;
    p_s[warp * kDecodeChunk + lane] = p;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < PPL; ++i) {
      acc[i].x *= corr;
      acc[i].y *= corr;
    }
    // weighted values: lane owns bf16 pairs lane, lane + 32, ...
#pragma unroll 4
    for (int j = 0; j < n; ++j) {
      const float pj = p_s[warp * kDecodeChunk + j];
#pragma unroll
      for (int i = 0; i < PPL; ++i) {
        const int pr = lane + 32 * i;
        if (NP % 32 == 0 || pr < NP) {
          const uint32_t v2 = vw32[j * NVP * 4 + pr];
          acc[i].x = fmaf(pj, __uint_as_float(v2 << 16), acc[i].x);
          acc[i].y = fmaf(pj, __uint_as_float(v2 & 0xffff0000u), acc[i].y);
        }
      }
    }
  }

  const size_t ob = ((size_t)b * a.H + h) * D;
  auto write_out = [&](const float2* o, float inv) {
#pragma unroll
    for (int i = 0; i < PPL; ++i) {
      const int pr = lane + 32 * i;
      if (NP % 32 != 0 && pr >= NP) continue;
      if (a.out_f32)
        reinterpret_cast<float2*>(static_cast<float*>(a.out) + ob)[pr] =
            make_float2(o[i].x * inv, o[i].y * inv);
      else
        reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(a.out) + ob)[pr] =
            __floats2bfloat162_rn(o[i].x * inv, o[i].y * inv);
    }
  };
  if (busy == 1) {  // the whole window in this CTA
    write_out(acc, 1.0f / l);
    return;
  }
  float* ph = a.part + ((size_t)b * a.H + h) * a.slots * (D + 2);
  float* part = ph + (size_t)slot * (D + 2);
#pragma unroll
  for (int i = 0; i < PPL; ++i) {
    const int pr = lane + 32 * i;
    if (NP % 32 == 0 || pr < NP) reinterpret_cast<float2*>(part)[pr] = acc[i];
  }
  if (lane == 0) {
    part[D] = m;
    part[D + 1] = l;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* cnt = a.counters + (size_t)b * a.KVH + kvh;
    const int last = atomicAdd(cnt, 1) == busy - 1;
    if (last) *cnt = 0;  // every CTA of the group has arrived: ready for the next launch
    last_s = last;
  }
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  // the last CTA merges its group's heads, slots in order
  float mx = -INFINITY;
  for (int t = 0; t < busy; ++t) mx = fmaxf(mx, __ldcg(ph + (size_t)t * (D + 2) + D));
  float2 o[PPL];
#pragma unroll
  for (int i = 0; i < PPL; ++i) o[i] = make_float2(0.f, 0.f);
  float L = 0.f;
  for (int t = 0; t < busy; ++t) {
    const float* pt = ph + (size_t)t * (D + 2);
    const float w = __expf(__ldcg(pt + D) - mx);
    L = fmaf(w, __ldcg(pt + D + 1), L);
#pragma unroll
    for (int i = 0; i < PPL; ++i) {
      const int pr = lane + 32 * i;
      if (NP % 32 == 0 || pr < NP) {
        const float2 v = __ldcg(reinterpret_cast<const float2*>(pt) + pr);
        o[i].x = fmaf(w, v.x, o[i].x);
        o[i].y = fmaf(w, v.y, o[i].y);
      }
    }
  }
  write_out(o, 1.0f / L);
}

int decode_attn_chunks(int max_positions) {
  return (max_positions + kDecodeChunk - 1) / kDecodeChunk;
}

// CTAs per (batch row, kv head): about 256 / B, at most one per chunk.
int decode_attn_slots(int batch, int max_positions) {
  const int want = batch > 0 ? max(1, 256 / batch) : 1;
  return min(decode_attn_chunks(max_positions), want);
}

template <int D, int G>
static int launch_decode_dg(const DecodeAttnArgs& a, cudaStream_t stream) {
  const size_t smem = (size_t)kDecodeChunk * ((D / 8) | 1) * 16 * (a.v_cache != nullptr ? 2 : 1) +
                      (size_t)G * D * 4 + (size_t)G * kDecodeChunk * 4;
  return launch_pdl(decode_attn_kernel<D, G>, dim3(a.slots, a.KVH, a.B), dim3(32 * G), smem,
                    stream, a) == cudaSuccess
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
