// Multi-token LoRA linear (batched decode and prefill chunks, 9..128 tokens)
// on the 5th-generation tensor cores, plus the small activation kernels that
// feed it.
//
// pl_linear_lora_gemm computes y[t, n] = epilogue(sum_k x[t, k] * w[n, k])
// for T <= 128 tokens.  A CTA owns a 128-row tile of the weight matrix and a
// contiguous range of 64-column K chunks.  One thread streams the weight tile
// (128 x 64 bf16, 16 KB) and the activation tile (N x 64) of each chunk into a
// shared-memory ring with 2-D TMA (128-byte swizzle); one thread issues
// tcgen05.mma (M = 128 weight rows, N = tokens padded to 16/32/64/128, K = 16)
// with the accumulator in tensor memory; then all four warps read the
// accumulator back with tcgen05.ld (warp w owns rows 32w..32w+31) and run the
// same epilogue as the decode GEMV (bias, per-token LoRA expand with its
// adapter, residual; the reference's bf16 rounding points).
//
// When the row tiles alone cannot fill the device, K is split across CTAs:
// every split writes its fp32 tile to the workspace and the last split to
// arrive (ticket per tile) adds the splits in split order -- deterministic --
// and runs the epilogue.  No device-side wait depends on another CTA.
#include "pl_linear_common.cuh"

#include <mutex>

namespace pl {

constexpr int kGemmM = 128;      // weight rows per tile (UMMA M)
constexpr int kGemmKC = 64;      // K per stage: one 128-byte swizzled row of bf16
constexpr int kGemmThreads = 128;

struct GemmArgs {
  GemvArgs e;          // epilogue fields: n_out, bias, LoRA, residual, y, status; T, K
  int32_t num_chunks;  // ceil(K / 64)
  int32_t num_splits;
  int32_t stages;
  float* partial;      // [m_tiles][splits][N][128] fp32 (num_splits > 1)
  int32_t* counters;   // [m_tiles] arrival tickets, zero between calls
};

template <int N>
struct GemmCfg {
  static constexpr int kABytes = kGemmM * 128;  // 16 KB weight tile
  static constexpr int kBBytes = N * 128;       // activation tile
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = N < 32 ? 32 : N;
  static_assert(kBBytes % 1024 == 0, "swizzle atoms must stay 1024-byte aligned");
};

__host__ __device__ inline int gemm_smem_bytes(int stage_bytes, int stages) {
  return 1024 + stages * stage_bytes + (2 * stages + 1) * 8 + 32;
}

template <int N>
__global__ void __launch_bounds__(kGemmThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                     const GemmArgs g) {
  using C = GemmCfg<N>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = g.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * C::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* done = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int32_t* flags = reinterpret_cast<volatile int32_t*>(tmem_slot + 1);  // abort, last, issued, consumed

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int mt = blockIdx.x, split = blockIdx.y;
  const int c0 = split * g.num_chunks / g.num_splits;
  const int c1 = (split + 1) * g.num_chunks / g.num_splits;
  const int nc = c1 - c0;  // >= 1: the host keeps num_splits <= num_chunks

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    flags[0] = flags[1] = flags[2] = flags[3] = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  if (threadIdx.x == 32) {
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&xmap);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (threadIdx.x == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol = l2_evict_first_policy();
    const int pre = g.e.early_weights ? (nc < S ? nc : S) : 0;
    for (int i = 0; i < pre; ++i) {  // weights are not produced upstream: start them now
      mbar_arrive_expect_tx(&full[i], C::kStageBytes);
      tma_load_2d(smem + i * C::kStageBytes, &wmap, (c0 + i) * kGemmKC, mt * kGemmM, &full[i], pol);
    }
    pdl_wait();
    int i = 0;
    for (; i < nc; ++i) {
      const int s = i % S;
      if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1)) {
        set_status(g.e.status, PL_ERR_TIMEOUT);
        flags[0] = 1;
        break;
      }
      uint8_t* st = smem + s * C::kStageBytes;
      if (i >= pre) {
        mbar_arrive_expect_tx(&full[s], C::kStageBytes);
        tma_load_2d(st, &wmap, (c0 + i) * kGemmKC, mt * kGemmM, &full[s], pol);
      }
      tma_load_2d(st + C::kABytes, &xmap, (c0 + i) * kGemmKC, 0, &full[s], 0ull);
    }
    flags[2] = i > pre ? i : pre;
  } else if (threadIdx.x == 32) {
    // ---------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = umma_idesc_bf16(kGemmM, N);
    int i = 0;
    for (; i < nc; ++i) {
      const int s = i % S;
      if (!mbar_wait(&full[s], (i / S) & 1)) {
        set_status(g.e.status, PL_ERR_TIMEOUT);
        flags[0] = 1;
        break;
      }
      tc_fence_after();
      const uint32_t a0 = smem_u32(smem + s * C::kStageBytes);
      const uint32_t b0 = a0 + C::kABytes;
#pragma unroll
      for (int k = 0; k < kGemmKC / 16; ++k)
        umma_bf16(tmem, umma_desc_k_sw128(a0 + 32 * k), umma_desc_k_sw128(b0 + 32 * k), idesc,
                  (i > 0 || k > 0) ? 1u : 0u);
      umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
    }
    flags[3] = i;
    umma_commit(done);
  }

  // ------------------------------------------------------------ epilogue
  pdl_wait();  // residual, LoRA down and adapter ids come from upstream kernels
  if (!mbar_wait(done, 0)) {
    set_status(g.e.status, PL_ERR_TIMEOUT);
    flags[0] = 1;
  }
  tc_fence_after();
  __syncthreads();
  const bool abort = flags[0] != 0;
  const int row = 32 * warp + lane;
  const int64_t o = (int64_t)mt * kGemmM + row;
  const uint32_t lane_addr = tmem + ((uint32_t)(32 * warp) << 16);
  const int T = g.e.T;
  const bool row_ok = o < g.e.n_out;
  if (g.num_splits == 1) {
#pragma unroll 1
    for (int c = 0; c < N / 16; ++c) {
      float v[16];
      tmem_ld16(lane_addr + 16 * c, v);  // whole warp, whatever the row
      if (!abort && row_ok) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (16 * c + j < T) gemv_epilogue(g.e, o, 16 * c + j, v[j]);
      }
    }
  } else {
    float* mine = g.partial + ((int64_t)mt * g.num_splits + split) * N * kGemmM;
#pragma unroll 1
    for (int c = 0; c < N / 16; ++c) {
      float v[16];
      tmem_ld16(lane_addr + 16 * c, v);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (16 * c + j < T) __stcg(mine + (16 * c + j) * kGemmM + row, v[j]);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const int32_t ticket = atomicAdd(&g.counters[mt], 1);
      flags[1] = ticket == g.num_splits - 1 ? 1 : 0;
    }
    __syncthreads();
    if (flags[1]) {
      // Last split of this tile: add the splits in order, then the epilogue.
      __threadfence();
      const float* base = g.partial + (int64_t)mt * g.num_splits * N * kGemmM + row;
      const int S2 = g.num_splits;
#pragma unroll 1
      for (int t0 = 0; t0 < T; t0 += 8) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int s = 0; s < S2; ++s) {
          float p[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            p[j] = (t0 + j < T) ? __ldcg(base + ((int64_t)s * N + t0 + j) * kGemmM) : 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += p[j];
        }
        if (!abort && row_ok) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (t0 + j < T) gemv_epilogue(g.e, o, t0 + j, acc[j]);
        }
      }
      if (threadIdx.x == 0) g.counters[mt] = 0;
    }
  }

  // ------------------------------------------------------------ teardown
  if (threadIdx.x == 0) {
    // Loads issued but never consumed (abort only) must land before exit.
    const int issued = flags[2], consumed = flags[3];
    for (int i = consumed; i < issued; ++i) (void)mbar_wait(&full[i % S], (i / S) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// -------------------------------------------------- activation prologues
// FlashInfer RMSNorm (one rounding): y = bf16(x * rsqrt(mean(x^2) + eps) * w).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const bf16* __restrict__ x, int64_t x_stride, int K,
                                                      const bf16* __restrict__ w, float eps, bf16* __restrict__ y,
                                                      int64_t y_stride) {
  __shared__ float part[8];
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const bf16* xr = x + (int64_t)t * x_stride;
  float ss = 0.f;
  for (int k = threadIdx.x * 8; k < K; k += 256 * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(u[q]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += part[i];
  const float r = rsqrtf(tot / (float)K + eps);
  for (int k = threadIdx.x * 8; k < K; k += 256 * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + k);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
    const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv);
    uint4 out;
    uint32_t* uo = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(u[q]);
      const float2 gw = unpack_bf16x2(uw[q]);
      uo[q] = pack_bf16x2(f.x * r * gw.x, f.y * r * gw.y);
    }
    *reinterpret_cast<uint4*>(y + (int64_t)t * y_stride + k) = out;
  }
}

// y[t, k] = bf16(silu(x[t, k]) * x[t, K + k]) over a packed [gate | up] row.
__global__ void __launch_bounds__(256) silu_mul_kernel(const bf16* __restrict__ x, int64_t x_stride, int K,
                                                       bf16* __restrict__ y, int64_t y_stride) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.y;
  const bf16* xr = x + (int64_t)t * x_stride;
  for (int k = (blockIdx.x * 256 + threadIdx.x) * 8; k < K; k += gridDim.x * 256 * 8) {
    const uint4 gv = *reinterpret_cast<const uint4*>(xr + k);
    const uint4 uv = *reinterpret_cast<const uint4*>(xr + K + k);
    const uint32_t* ug = reinterpret_cast<const uint32_t*>(&gv);
    const uint32_t* uu = reinterpret_cast<const uint32_t*>(&uv);
    uint4 out;
    uint32_t* uo = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 gg = unpack_bf16x2(ug[q]);
      const float2 up = unpack_bf16x2(uu[q]);
      uo[q] = pack_bf16x2(silu_mul(gg.x, up.x), silu_mul(gg.y, up.y));
    }
    *reinterpret_cast<uint4*>(y + (int64_t)t * y_stride + k) = out;
  }
}

}  // namespace pl

// =================================================================== host
namespace {

struct Map2Key {
  const void* ptr;
  int64_t inner, rows, stride;
  int32_t box_rows, dev;
  bool operator==(const Map2Key& o) const {
    return ptr == o.ptr && inner == o.inner && rows == o.rows && stride == o.stride && box_rows == o.box_rows &&
           dev == o.dev;
  }
};
constexpr int kMap2Cache = 512;
struct Map2Cache {
  std::mutex mu;
  Map2Key key[kMap2Cache];
  CUtensorMap map[kMap2Cache];
  int used = 0, next = 0;
};
Map2Cache g_map2;

// bf16 matrix [rows][inner] with row stride `stride` elements; box 64 x box_rows,
// 128-byte swizzle, out-of-range rows/columns read as zero.
int32_t matrix_map(const void* ptr, int64_t inner, int64_t rows, int64_t stride, int box_rows, CUtensorMap* out) {
  int dev = 0;
  cudaGetDevice(&dev);
  Map2Key k{ptr, inner, rows, stride, box_rows, dev};
  std::lock_guard<std::mutex> lock(g_map2.mu);
  for (int i = 0; i < g_map2.used; ++i)
    if (g_map2.key[i] == k) {
      *out = g_map2.map[i];
      return PL_OK;
    }
  pl_host::EncodeTiledFn enc = pl_host::encode_tiled_fn();
  if (enc == nullptr) return PL_ERR_CUDA;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)pl::kGemmKC, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return PL_ERR_INVALID_ARGUMENT;
  int slot;
  if (g_map2.used < kMap2Cache) {
    slot = g_map2.used++;
  } else {
    slot = g_map2.next;
    g_map2.next = (g_map2.next + 1) % kMap2Cache;
  }
  g_map2.key[slot] = k;
  g_map2.map[slot] = m;
  *out = m;
  return PL_OK;
}

int gemm_n(int tokens) { return tokens <= 16 ? 16 : tokens <= 32 ? 32 : tokens <= 64 ? 64 : 128; }

int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

struct GemmShape {
  int n, stages, m_tiles, chunks, splits, stage_bytes;
};

GemmShape gemm_shape(int tokens, int k_in, int n_out, int sms) {
  GemmShape s;
  s.n = gemm_n(tokens);
  s.stage_bytes = pl::kGemmM * 128 + s.n * 128;
  s.m_tiles = (n_out + pl::kGemmM - 1) / pl::kGemmM;
  s.chunks = (k_in + pl::kGemmKC - 1) / pl::kGemmKC;
  // One CTA per SM; K is split only when the row tiles leave SMs idle, and
  // every split keeps at least 4 chunks.
  int splits = s.m_tiles >= sms ? 1 : sms / s.m_tiles;
  const int max_by_k = s.chunks / 4 > 0 ? s.chunks / 4 : 1;
  if (splits > max_by_k) splits = max_by_k;
  if (splits > 16) splits = 16;
  s.splits = splits < 1 ? 1 : splits;
  int stages = (200 * 1024) / s.stage_bytes;
  if (stages > 8) stages = 8;
  if (stages > s.chunks) stages = s.chunks < 2 ? 2 : s.chunks;
  s.stages = stages;
  return s;
}

int64_t gemm_workspace_bytes(const GemmShape& s) {
  int64_t b = align256((int64_t)s.m_tiles * 4);
  if (s.splits > 1) b += (int64_t)s.m_tiles * s.splits * s.n * pl::kGemmM * 4;
  return b;
}

template <int N>
int32_t launch_gemm(const CUtensorMap& wm, const CUtensorMap& xm, const pl::GemmArgs& g, int m_tiles, int splits,
                    int stage_bytes, int stages, void* stream) {
  auto kern = pl::linear_tc_kernel<N>;
  const int smem = pl::gemm_smem_bytes(stage_bytes, stages);
  int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  if (st != PL_OK) return st;
  return pl_host::launch_pdl(kern, dim3(m_tiles, splits), dim3(pl::kGemmThreads), smem, stream, wm, xm, g);
}

}  // namespace

extern "C" int32_t pl_linear_gemm_plan(int32_t num_tokens, int32_t k_in, int32_t n_out, pl_gemm_plan_t* plan) {
  if (plan == nullptr || num_tokens < 1 || num_tokens > 128 || k_in <= 0 || n_out <= 0) return PL_ERR_INVALID_ARGUMENT;
  int sms = pl_host::sm_count();
  if (sms <= 0) sms = 148;
  const GemmShape s = gemm_shape(num_tokens, k_in, n_out, sms);
  plan->num_splits = s.splits;
  plan->ctas = s.m_tiles * s.splits;
  plan->workspace_bytes = gemm_workspace_bytes(s);
  return PL_OK;
}

extern "C" int32_t pl_linear_lora_gemm(const void* x, int64_t x_stride, int32_t num_tokens, int32_t k_in,
                                       const void* w, int32_t n_out, const void* bias, const float* lora_down,
                                       int64_t down_stride, const void* lora_b, int32_t lora_rank, float lora_scale,
                                       const int32_t* slice_end, int32_t num_slices, const int32_t* tok_adapter,
                                       const void* residual, int64_t res_stride, void* y, int64_t y_stride,
                                       int32_t num_splits, void* workspace, int64_t workspace_bytes, int32_t flags,
                                       int32_t* status_dev, void* stream) {
  if (num_tokens == 0 || n_out == 0) return PL_OK;
  if (x == nullptr || w == nullptr || y == nullptr || num_tokens < 0 || num_tokens > 128 || k_in <= 0 ||
      n_out < 0 || workspace == nullptr)
    return PL_ERR_INVALID_ARGUMENT;
  if (k_in % 8 != 0 || x_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15))
    return PL_ERR_UNSUPPORTED;
  if (lora_b != nullptr && (lora_down == nullptr || lora_rank <= 0 || num_slices < 1 || num_slices > 4 ||
                            (num_slices > 1 && slice_end == nullptr)))
    return PL_ERR_INVALID_ARGUMENT;
  int sms = pl_host::sm_count();
  if (sms <= 0) sms = 148;
  const GemmShape s = gemm_shape(num_tokens, k_in, n_out, sms);
  if (num_splits < 1 || num_splits > s.chunks || num_splits > 16) return PL_ERR_INVALID_ARGUMENT;
  GemmShape sh = s;
  sh.splits = num_splits;
  if (workspace_bytes < gemm_workspace_bytes(sh) || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return PL_ERR_WORKSPACE_TOO_SMALL;

  CUtensorMap wm, xm;
  int32_t st = matrix_map(w, k_in, n_out, k_in, pl::kGemmM, &wm);
  if (st != PL_OK) return st;
  st = matrix_map(x, k_in, num_tokens, x_stride, sh.n, &xm);
  if (st != PL_OK) return st;

  pl::GemmArgs g = {};
  pl::GemvArgs& a = g.e;
  a.x = static_cast<const pl::bf16*>(x);
  a.x_stride = x_stride;
  a.T = num_tokens;
  a.K = k_in;
  a.w = static_cast<const pl::bf16*>(w);
  a.n_out = n_out;
  a.bias = static_cast<const pl::bf16*>(bias);
  a.lora_down = lora_down;
  a.down_stride = down_stride;
  a.lora_b = static_cast<const pl::bf16*>(lora_b);
  a.rank = lora_rank;
  a.lora_scale = lora_scale;
  a.num_slices = num_slices < 1 ? 1 : num_slices;
  for (int i = 0; i < 4; ++i) a.slice_end[i] = n_out;
  for (int i = 0; i < num_slices - 1 && slice_end != nullptr; ++i) a.slice_end[i] = slice_end[i];
  a.tok_adapter = tok_adapter;
  a.residual = static_cast<const pl::bf16*>(residual);
  a.res_stride = res_stride;
  a.y = static_cast<pl::bf16*>(y);
  a.y_stride = y_stride;
  a.early_weights = (flags & PL_FLAG_WEIGHTS_STATIC) ? 1 : 0;
  a.status = status_dev;
  g.num_chunks = sh.chunks;
  g.num_splits = num_splits;
  g.stages = sh.stages;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  g.counters = reinterpret_cast<int32_t*>(ws);
  g.partial = num_splits > 1 ? reinterpret_cast<float*>(ws + align256((int64_t)sh.m_tiles * 4)) : nullptr;

  switch (sh.n) {
    case 16: return launch_gemm<16>(wm, xm, g, sh.m_tiles, num_splits, sh.stage_bytes, sh.stages, stream);
    case 32: return launch_gemm<32>(wm, xm, g, sh.m_tiles, num_splits, sh.stage_bytes, sh.stages, stream);
    case 64: return launch_gemm<64>(wm, xm, g, sh.m_tiles, num_splits, sh.stage_bytes, sh.stages, stream);
    default: return launch_gemm<128>(wm, xm, g, sh.m_tiles, num_splits, sh.stage_bytes, sh.stages, stream);
  }
}

extern "C" int32_t pl_rmsnorm(const void* x, int64_t x_stride, int32_t num_tokens, int32_t k_in, const void* w,
                              float eps, void* y, int64_t y_stride, void* stream) {
  if (num_tokens == 0) return PL_OK;
  if (x == nullptr || w == nullptr || y == nullptr || num_tokens < 0 || k_in <= 0) return PL_ERR_INVALID_ARGUMENT;
  if (k_in % 8 || x_stride % 8 || y_stride % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return PL_ERR_UNSUPPORTED;
  return pl_host::launch_pdl(pl::rmsnorm_kernel, dim3(num_tokens), dim3(256), 0, stream,
                             static_cast<const pl::bf16*>(x), x_stride, (int)k_in, static_cast<const pl::bf16*>(w),
                             eps, static_cast<pl::bf16*>(y), y_stride);
}

extern "C" int32_t pl_silu_mul(const void* x, int64_t x_stride, int32_t num_tokens, int32_t k_out, void* y,
                               int64_t y_stride, void* stream) {
  if (num_tokens == 0) return PL_OK;
  if (x == nullptr || y == nullptr || num_tokens < 0 || num_tokens > 65535 || k_out <= 0)
    return PL_ERR_INVALID_ARGUMENT;
  if (k_out % 8 || x_stride % 8 || y_stride % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(y) & 15))
    return PL_ERR_UNSUPPORTED;
  int blocks = (k_out / 8 + 255) / 256;
  if (blocks > 64) blocks = 64;
  return pl_host::launch_pdl(pl::silu_mul_kernel, dim3(blocks, num_tokens), dim3(256), 0, stream,
                             static_cast<const pl::bf16*>(x), x_stride, (int)k_out, static_cast<pl::bf16*>(y),
                             y_stride);
}
