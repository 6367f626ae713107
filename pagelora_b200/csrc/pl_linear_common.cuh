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
};

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
  if (a.residual != nullptr) v = bf2f(a.residual[tok * a.res_stride + o]) + bfr(v);
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
__device__ __forceinline__ void epilogue_rows4(const GemvArgs& a, int64_t o0, int tok, const float* v) {
  if (o0 >= a.n_out) return;
  bf16* dst = a.y + tok * a.y_stride + o0;
  if (o0 + 4 <= a.n_out && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
    float r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = epilogue_value(a, o0 + i, tok, v[i]);
    *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]));
  } else {
    for (int i = 0; i < 4 && o0 + i < a.n_out; ++i) dst[i] = f2bf(epilogue_value(a, o0 + i, tok, v[i]));
  }
}

}  // namespace pl
