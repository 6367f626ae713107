// Per-head transform of the packed [q | k | v] projection row of one token,
// shared by the standalone q/k/v kernel and the fused decode-attention
// kernel: LoRA-B expand (the packed delta of model/flashinfer/packed_ops.py
// :314-384 with bf16 rounding of the projection, of the delta and of the
// sum), Qwen3 head RMSNorm as the Hugging Face module computes it (fp32
// normalise, round, scale, round; model/flashinfer/projection.py:90-103) and
// non-interleaved RoPE in fp32 (projection.py:155-190).
#pragma once

#include "pl_common.cuh"

namespace pl {

struct QkvHeadArgs {
  const bf16* qkv;          // [T, (Hq + 2 Hkv) * D] row stride qkv_stride
  int64_t qkv_stride;
  const float* down;        // [T, 3 * rank] LoRA-A products (q | k | v), nullable
  int64_t down_stride;
  const bf16* lora_b;       // [n_adapters, (Hq + 2 Hkv) * D, rank], nullable
  int32_t rank;
  float lora_scale;
  const int32_t* tok_adapter;  // nullable: adapter 0
  const bf16* q_norm_w;     // [D], nullable (no head norm)
  const bf16* k_norm_w;
  float eps;
  const int32_t* positions; // [T]
  float theta;
  const float* rope_cs;     // nullable: [T][D/2] (cos, sin) pairs of pl_rope_cos_sin; else computed here
  int32_t Hq, Hkv;
};

// cos and sin of RoPE angle i (0 <= i < D/2) at position pos, in fp32
// (non-interleaved rotation of projection.py:155-190).  The one definition
// used both by the per-step table kernel and by the inline path, so the two
// give identical values.
__device__ __forceinline__ void rope_angle_cs(float pos, int i, int D, float theta, float& cs, float& sn) {
  const float inv_freq = 1.0f / powf(theta, (float)(2 * i) / (float)D);
  sincosf(pos * inv_freq, &sn, &cs);
}

__device__ __forceinline__ void prefetch_l2_line(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// L2 prefetch of the operands of head `hh` that do not come from upstream
// kernels (the head-norm weights, and the LoRA B rows when every token uses
// adapter 0): issued before the grid dependency resolves, so that the
// transform afterwards finds them in L2.
template <int D>
__device__ __forceinline__ void qkv_head_prefetch(const QkvHeadArgs& a, int hh, int lane) {
  constexpr int E = D / 32;
  const int kind = hh < a.Hq ? 0 : (hh < a.Hq + a.Hkv ? 1 : 2);
  const int d0 = lane * E;
  if (a.lora_b != nullptr && a.down != nullptr && a.tok_adapter == nullptr) {
    const bf16* b0 = a.lora_b + ((int64_t)hh * D + d0) * a.rank;
    for (int off = 0; off < E * a.rank; off += 64) prefetch_l2_line(b0 + off);  // 128-byte lines
  }
  const bf16* nw = kind == 0 ? a.q_norm_w : (kind == 1 ? a.k_norm_w : nullptr);
  if (nw != nullptr && (lane & 15) == 0) prefetch_l2_line(nw + d0);
}

// One warp: head `hh` (q heads, then k heads, then v heads) of token t.
// Lane l holds elements [l * E, l * E + E), E = D / 32 (lanes 0..15 the
// first half of the head, 16..31 the second, which RoPE pairs).  Every
// operand load that does not depend on another is issued up front, so the
// transform costs about two memory round trips.
template <int D>
__device__ __forceinline__ void qkv_head_transform(const QkvHeadArgs& a, int t, int hh, int lane, float* v,
                                                   bool trace = false) {
  constexpr int E = D / 32;
  const int kind = hh < a.Hq ? 0 : (hh < a.Hq + a.Hkv ? 1 : 2);  // q, k, v
  const int col = hh * D;                                          // packed column of this head
  const int d0 = lane * E;
  const bool lora = a.down != nullptr && a.lora_b != nullptr;
  const bf16* nw = kind == 0 ? a.q_norm_w : (kind == 1 ? a.k_norm_w : nullptr);
  // independent loads first: the projection row, the position, the adapter
  // id, the norm weights, the RoPE (cos, sin) pairs of the step's table
  {
    const bf16* src = a.qkv + (int64_t)t * a.qkv_stride + col + d0;
    if constexpr (E == 4) {
      if ((reinterpret_cast<uintptr_t>(src) & 7) == 0) {
        const uint2 u = *reinterpret_cast<const uint2*>(src);
        const float2 f0 = unpack_bf16x2(u.x), f1 = unpack_bf16x2(u.y);
        v[0] = f0.x;
        v[1] = f0.y;
        v[2] = f1.x;
        v[3] = f1.y;
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) v[e] = bf2f(src[e]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = bf2f(src[e]);
    }
  }
  const float pos = (kind < 2 && a.rope_cs == nullptr) ? (float)a.positions[t] : 0.f;
  const int ad = (lora && a.tok_adapter != nullptr) ? a.tok_adapter[t] : 0;
  float wn[E];
#pragma unroll
  for (int e = 0; e < E; ++e) wn[e] = nw != nullptr ? bf2f(nw[d0 + e]) : 1.f;
  float csn[2 * E];  // (cos, sin) of the E rotation angles of this lane
  if (kind < 2 && a.rope_cs != nullptr) {
    const float* src = a.rope_cs + ((int64_t)t * (D / 2) + d0 % (D / 2)) * 2;
#pragma unroll
    for (int e = 0; e < 2 * E; e += 4) *reinterpret_cast<float4*>(csn + e) = *reinterpret_cast<const float4*>(src + e);
  }
  if (trace && lane == 0) {
    asm volatile("" ::"f"(v[0]), "f"(pos), "f"(wn[0]), "r"(ad));
    PL_TRACE_POINT(10);
  }
  if (lora && ad >= 0) {
    const int n_out = (a.Hq + 2 * a.Hkv) * D;
    const float* drow = a.down + (int64_t)t * a.down_stride + kind * a.rank;
    const bf16* brow0 = a.lora_b + ((int64_t)ad * n_out + col + d0) * a.rank;  // E consecutive rows
    float d[E];
    if (a.rank == 16 && ((reinterpret_cast<uintptr_t>(brow0) | reinterpret_cast<uintptr_t>(drow)) & 15) == 0) {
      // rank 16: every B and down element requested before any arithmetic
      uint4 bq[2 * E];
      float4 dq[4];
#pragma unroll
      for (int i = 0; i < 2 * E; ++i) bq[i] = reinterpret_cast<const uint4*>(brow0)[i];
#pragma unroll
      for (int i = 0; i < 4; ++i) dq[i] = reinterpret_cast<const float4*>(drow)[i];
      float dr[16];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        dr[4 * i] = bfr(dq[i].x);
        dr[4 * i + 1] = bfr(dq[i].y);
        dr[4 * i + 2] = bfr(dq[i].z);
        dr[4 * i + 3] = bfr(dq[i].w);
      }
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float acc = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t* u = reinterpret_cast<const uint32_t*>(&bq[2 * e + h]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = unpack_bf16x2(u[q]);
            acc = fmaf(f.x, dr[8 * h + 2 * q], acc);
            acc = fmaf(f.y, dr[8 * h + 2 * q + 1], acc);
          }
        }
        d[e] = acc;
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) d[e] = lora_dot(brow0 + e * a.rank, drow, a.rank);
    }
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = bfr(v[e] + bfr(bfr(d[e]) * a.lora_scale));
  }
  if (trace && lane == 0) {
    asm volatile("" ::"f"(v[0]));
    PL_TRACE_POINT(14);
  }
  if (kind < 2) {
    if (nw != nullptr) {  // HF RMSNorm module: fp32 normalise, round, scale, round
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) ss += v[e] * v[e];
      ss = warp_sum(ss);
      const float r = rsqrtf(ss / (float)D + a.eps);
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = bfr(wn[e] * bfr(v[e] * r));
    }
    if (trace && lane == 0) {
      asm volatile("" ::"f"(v[0]));
      PL_TRACE_POINT(15);
    }
    float out[E];
    if (a.rope_cs == nullptr) {
#pragma unroll
      for (int e = 0; e < E; ++e) rope_angle_cs(pos, (d0 + e) % (D / 2), D, a.theta, csn[2 * e], csn[2 * e + 1]);
    }
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
      const float cs = csn[2 * e], sn = csn[2 * e + 1];
      out[e] = lane < 16 ? v[e] * cs - partner * sn : v[e] * cs + partner * sn;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = out[e];
  }
}

}  // namespace pl
