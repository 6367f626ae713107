// Shared pieces of the linear-layer kernels: the argument block and the
// per-element epilogue (bias, LoRA expand, residual) with the reference's
// bf16 rounding points.
#pragma once

#include "pl_common.cuh"

namespace pl {

constexpr int kTileRows = 16;  // rows per tile (mma M)
constexpr int kMaxTok = 8;     // mma N

struct GemvArgs {
  const bf16* x;
  int64_t x_stride;
  int32_t T, K;
  int32_t prologue;
  const bf16* norm_w;
  float eps;
  const bf16* w;
  int32_t n_out;
  const bf16* bias;
  const float* lora_down;
  int64_t down_stride;
  const bf16* lora_b;
  int32_t rank;
  float lora_scale;
  int32_t slice_end[4];
  int32_t num_slices;
  const int32_t* tok_adapter;
  const bf16* residual;
  int64_t res_stride;
  bf16* y;
  int64_t y_stride;
  const bf16* shrink_a;
  int32_t n_shrink;
  const bf16* pro_a;      // LoRA A stack [adapters][rank][K]: down computed in the kernel from x (or null)
  int32_t pro_a_adapters;
  float* shrink_out;
  int64_t shrink_stride;
  int32_t early_weights;  // weights are not produced upstream: stream them before the dependency resolves
  int32_t stages;         // depth of the shared-memory ring
  int32_t kc;             // columns per stage (multiple of 16)
  int32_t prefetch_tiles; // tiles per CTA whose weights are pulled into L2 before the dependency resolves
  int32_t* status;
  // L2 prefetch of the next projection's first ring stages (pl_linear_lora_phase): weight rows
  // [n_out) from pf_w, rows past it from pf_shrink, split over pf_grid CTAs as that launch splits them
  const bf16* pf_w;
  const bf16* pf_shrink;
  int64_t pf_rows_total;
  int32_t pf_n_out, pf_k, pf_kc, pf_units, pf_grid;
  int32_t silu_pairs;     // GEMM: 128-row tiles of 64 gate rows then the 64 matching up rows; y = the SiLU-and-mul
  int32_t coherent;       // activations / residual may have been written by other CTAs of this launch: read them
                          // from L2 (ld.global.cg), never from a possibly stale L1 line
};

// 16 activation bytes; from L2 when kCg (data written by other CTAs of the same launch).
template <bool kCg>
__device__ __forceinline__ uint4 ld_act16(const void* p) {
  if constexpr (kCg) {
    return __ldcg(reinterpret_cast<const uint4*>(p));
  } else {
    return *reinterpret_cast<const uint4*>(p);
  }
}

__device__ __forceinline__ bf16 ld_bf16_cg(const bf16* p) {
  unsigned short u;
  asm volatile("ld.global.cg.u16 %0, [%1];" : "=h"(u) : "l"(p));
  return __ushort_as_bfloat16(u);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.f + expf(-g)) * u; }

// Epilogue value of one output element (row o < n_out, token tok) from its
// fp32 dot product: bias, LoRA expand, residual, with the reference's bf16
// rounding points (the caller rounds the result to bf16 once more).
// `down` / `dstride`: the LoRA down rows (a.lora_down, or the kernel's own
// copy in shared memory).
__device__ __forceinline__ float epilogue_value(const GemvArgs& a, int64_t o, int tok, float v, const float* down,
                                                int64_t dstride) {
  if (a.bias != nullptr) v += bf2f(a.bias[o]);
  if (a.lora_b != nullptr) {
    const int ad = a.tok_adapter != nullptr ? a.tok_adapter[tok] : 0;
    float vb = bfr(v);
    if (ad >= 0) {
      int sl = 0;
      while (sl < a.num_slices - 1 && o >= a.slice_end[sl]) ++sl;
      const bf16* brow = a.lora_b + ((int64_t)ad * a.n_out + o) * a.rank;
      const float* drow = down + tok * dstride + sl * a.rank;
      const float d = lora_dot(brow, drow, a.rank);
      vb = bfr(vb + bfr(bfr(d) * a.lora_scale));
    }
    v = vb;
  }
  if (a.residual != nullptr) {
    const bf16* rp = a.residual + tok * a.res_stride + o;
    v = bf2f(a.coherent ? ld_bf16_cg(rp) : *rp) + bfr(v);
  }
  return v;
}

__device__ __forceinline__ float epilogue_value(const GemvArgs& a, int64_t o, int tok, float v) {
  return epilogue_value(a, o, tok, v, a.lora_down, a.down_stride);
}

// Epilogue of one output element (row o, token tok): rows past n_out are
// LoRA-A shrink rows whose fp32 products go to shrink_out.
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int64_t o, int tok, float v, const float* down,
                                              int64_t dstride) {
  if (o >= a.n_out) {
    a.shrink_out[tok * a.shrink_stride + (o - a.n_out)] = v;
    return;
  }
  a.y[tok * a.y_stride + o] = f2bf(epilogue_value(a, o, tok, v, down, dstride));
}
__device__ __forceinline__ void gemv_epilogue(const GemvArgs& a, int64_t o, int tok, float v) {
  gemv_epilogue(a, o, tok, v, a.lora_down, a.down_stride);
}

// Epilogue of rows o0..o0+3 (o0 % 4 == 0) of one token, stored as one 8-byte
// vector when the four rows exist and the destination is 8-byte aligned.
// Rows at or past row_end (default: n_out) are left alone.
__device__ __forceinline__ void epilogue_rows4(const GemvArgs& a, int64_t o0, int tok, const float* v,
                                               int64_t row_end = -1) {
  if (row_end < 0 || row_end > a.n_out) row_end = a.n_out;
  if (o0 >= row_end) return;
  bf16* dst = a.y + tok * a.y_stride + o0;
  if (o0 + 4 <= row_end && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
    float r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = epilogue_value(a, o0 + i, tok, v[i]);
    *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]));
  } else {
    for (int i = 0; i < 4 && o0 + i < row_end; ++i) dst[i] = f2bf(epilogue_value(a, o0 + i, tok, v[i]));
  }
}

constexpr int kGemmTileRows = 128;  // weight rows of one tcgen05 GEMM tile

// SiLU-and-mul epilogue of GEMM tile `tile` whose rows [0, 64) are gate rows
// and [64, 128) the matching up rows (the gate/up weights interleaved in
// blocks of 64): lane l < 16 holds gate rows 4l .. 4l+3 of tokens tok[0..nt),
// lane l + 16 the up rows, which come over by a shuffle; then
// y[tok][64 * tile + 4l + i] = bf16(silu(bf16(g)) * bf16(u)), the rounding of
// a bf16 gate_up output followed by the SiLU-and-mul kernel.  Every lane of
// the warp calls it (full-mask shuffles).
__device__ __forceinline__ void epilogue_silu_pairs(const GemvArgs& a, int64_t tile, int lane, const int (&tok)[4],
                                                    int nt, const float (&v)[4][4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float up[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) up[i] = __shfl_down_sync(0xffffffffu, v[k][i], 16);
    if (lane < 16 && k < nt) {
      float r[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) r[i] = silu_mul(bfr(v[k][i]), bfr(up[i]));
      *reinterpret_cast<uint2*>(a.y + tok[k] * a.y_stride + 64 * tile + 4 * lane) =
          make_uint2(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]));
    }
  }
}

// Rank-16 LoRA dot product with the B row held in registers (16 bf16) and
// the down row already rounded to bf16: the fma order of lora_dot.
__device__ __forceinline__ float lora_dot16(const uint4 (&b)[2], const float* d) {
  float acc = 0.f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float4 d0 = *reinterpret_cast<const float4*>(d + 8 * h);
    const float4 d1 = *reinterpret_cast<const float4*>(d + 8 * h + 4);
    const float2 b0 = unpack_bf16x2(b[h].x), b1 = unpack_bf16x2(b[h].y), b2 = unpack_bf16x2(b[h].z),
                 b3 = unpack_bf16x2(b[h].w);
    acc = fmaf(b0.x, d0.x, acc);
    acc = fmaf(b0.y, d0.y, acc);
    acc = fmaf(b1.x, d0.z, acc);
    acc = fmaf(b1.y, d0.w, acc);
    acc = fmaf(b2.x, d1.x, acc);
    acc = fmaf(b2.y, d1.y, acc);
    acc = fmaf(b3.x, d1.z, acc);
    acc = fmaf(b3.y, d1.w, acc);
  }
  return acc;
}

// Epilogue of rows o0..o0+3 (o0 % 4 == 0) for the tokens tok[0..nt) (nt <= 4),
// with the values of epilogue_value.  Every input of the tokens (adapter ids,
// residuals, rank-16 LoRA rows) is loaded before the first result is formed
// and the results are stored last, so the tokens' memory latencies overlap
// instead of adding up.  Other shapes fall back to one token at a time.
// sdown / sad (optional, rank 16): the down rows [T][sR] rounded to bf16 and
// the adapter ids [T], staged in shared memory; each adapter's B rows are then
// loaded once for consecutive tokens that share it.
// sdelta (optional, with sad): the finished LoRA terms bf16(bf16(d) * scale)
// of this tile, [T][128] bf16 with row o0 at column o0 - sdelta_row0,
// computed ahead by the caller; they replace the expand here.
// Rows at or past row_end (default: n_out) are left alone.
__device__ __forceinline__ void epilogue_rows4_x4(const GemvArgs& a, int64_t o0, const int (&tok)[4], int nt,
                                                  const float (&v)[4][4], const float* sdown = nullptr,
                                                  int sR = 0, const int32_t* sad = nullptr,
                                                  const bf16* sdelta = nullptr, int64_t sdelta_row0 = 0,
                                                  int64_t row_end = -1) {
  if (row_end < 0 || row_end > a.n_out) row_end = a.n_out;
  if (o0 >= row_end) return;
  const bool vec = o0 + 4 <= row_end && (a.lora_b == nullptr || a.rank == 16) &&
                   ((a.y_stride | a.res_stride) & 3) == 0 &&
                   ((reinterpret_cast<uintptr_t>(a.y) | reinterpret_cast<uintptr_t>(a.residual)) & 7) == 0;
  if (!vec) {
    for (int k = 0; k < nt; ++k) epilogue_rows4(a, o0, tok[k], v[k], row_end);
    return;
  }
  float bias[4] = {0.f, 0.f, 0.f, 0.f};
  if (a.bias != nullptr) {
#pragma unroll
    for (int i = 0; i < 4; ++i) bias[i] = bf2f(a.bias[o0 + i]);
  }
  int ad[4] = {0, 0, 0, 0};
  if (a.lora_b != nullptr && sad != nullptr) {
#pragma unroll
    for (int k = 0; k < 4; ++k) ad[k] = k < nt ? sad[tok[k]] : -1;
  } else if (a.lora_b != nullptr && a.tok_adapter != nullptr) {
#pragma unroll
    for (int k = 0; k < 4; ++k) ad[k] = k < nt ? a.tok_adapter[tok[k]] : -1;
  }
  uint2 res[4] = {};
  if (a.residual != nullptr) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (k < nt) res[k] = *reinterpret_cast<const uint2*>(a.residual + tok[k] * a.res_stride + o0);
  }
  float dl[4][4] = {};
  if (a.lora_b != nullptr && sdelta != nullptr) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (k < nt) {
        const uint2 d2 = *reinterpret_cast<const uint2*>(sdelta + tok[k] * kGemmTileRows + (o0 - sdelta_row0));
        const float2 d01 = unpack_bf16x2(d2.x), d23 = unpack_bf16x2(d2.y);
        dl[k][0] = d01.x;
        dl[k][1] = d01.y;
        dl[k][2] = d23.x;
        dl[k][3] = d23.y;
      }
    }
  } else if (a.lora_b != nullptr) {
    int sl[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      sl[i] = 0;
      while (sl[i] < a.num_slices - 1 && o0 + i >= a.slice_end[sl[i]]) ++sl[i];
    }
    if (sdown != nullptr) {
      int cur = -1;  // adapter whose B rows are in b
      uint4 b[4][2] = {};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (k < nt && ad[k] >= 0) {
          if (ad[k] != cur) {
            cur = ad[k];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint4* br = reinterpret_cast<const uint4*>(a.lora_b + ((int64_t)cur * a.n_out + o0 + i) * 16);
              b[i][0] = br[0];
              b[i][1] = br[1];
            }
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) dl[k][i] = lora_dot16(b[i], sdown + tok[k] * sR + sl[i] * 16);
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (k < nt && ad[k] >= 0) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dl[k][i] = lora_dot(a.lora_b + ((int64_t)ad[k] * a.n_out + o0 + i) * 16,
                                a.lora_down + tok[k] * a.down_stride + sl[i] * 16, 16);
        }
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (k >= nt) continue;
    const float2 r01 = unpack_bf16x2(res[k].x), r23 = unpack_bf16x2(res[k].y);
    const float rv[4] = {r01.x, r01.y, r23.x, r23.y};
    float out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float x = v[k][i];
      if (a.bias != nullptr) x += bias[i];
      if (a.lora_b != nullptr) {
        float vb = bfr(x);
        if (ad[k] >= 0) vb = bfr(vb + (sdelta != nullptr ? dl[k][i] : bfr(bfr(dl[k][i]) * a.lora_scale)));
        x = vb;
      }
      if (a.residual != nullptr) x = rv[i] + bfr(x);
      out[i] = x;
    }
    *reinterpret_cast<uint2*>(a.y + tok[k] * a.y_stride + o0) =
        make_uint2(pack_bf16x2(out[0], out[1]), pack_bf16x2(out[2], out[3]));
  }
}

}  // namespace pl
