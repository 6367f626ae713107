// Multi-token LoRA linear (batched decode and prefill chunks, 1..128 tokens)
// on the 5th-generation tensor cores, plus the small activation kernels that
// feed it.
//
// pl_linear_lora_gemm computes y[t, n] = epilogue(sum_k x[t, k] * w[n, k]).
// CTA c of the grid owns the weight-row band [c*R, c*R + R) over the whole
// of K, so no output is shared between CTAs: nothing is merged, and the
// only tail after the last MMA is the band's own epilogue.  R is about
// n_out / SMs (a multiple of 4), cut into segments of at most 128 rows
// (one UMMA M tile, rows past the segment read as garbage and are never
// stored); every SM streams the same number of weight bytes.  Per CTA:
//   warp 0     streams each unit (one segment x one K block of kcs x 64
//              columns) as kcs 2-D TMA copies of the segment's rows plus
//              kcs copies of the activation chunk into a shared-memory
//              ring, several units per issuing instruction;
//   warp 1     (one lane) issues tcgen05.mma (M = 128, N = tokens padded to
//              16/32/64/128, K = 16) into one of two tensor-memory
//              accumulators, one per segment;
//   warps 2-5  read a finished accumulator with tcgen05.ld (warp w owns
//              lanes 32(w%4)..) while the next segment accumulates, and run
//              the decode GEMV's epilogue (bias, per-token LoRA expand with
//              the token's adapter, residual; the reference's bf16 rounding
//              points), staged through shared memory into 8-byte stores.
//              With rank-16 LoRA they first compute the LoRA terms of the
//              CTA's last segment while the weights stream.
#include "pl_linear_common.cuh"

#include <mutex>

namespace pl {

constexpr int kGemmM = 128;      // UMMA M: rows one accumulator holds
constexpr int kGemmKC = 64;      // K per chunk: one 128-byte swizzled row of bf16
constexpr int kGemmThreads = 192;
constexpr int kGemmIssue = 4;    // units per producer TMA instruction
constexpr int kGemmGuard = kGemmM * 128;  // MMA reads 128 rows from a slot: slack after the ring

struct GemmArgs {
  GemvArgs e;          // epilogue fields: n_out, bias, LoRA, residual, y, status; T, K
  int32_t kblocks;     // K blocks per segment
  int32_t band_rows;   // rows per CTA
  int32_t seg_rows;    // rows per segment (<= 128, a multiple of 4)
  int32_t nseg;        // segments per band
  int32_t a_slot;      // bytes of one weight chunk slot (seg_rows rounded up to 8, x 128 B)
  int32_t stage_bytes;
  int32_t stages;
  int32_t lora_stage;  // bytes of shared memory holding the rank-16 LoRA down rows and adapter ids (0: none)
  int32_t lora_delta;  // bytes holding the precomputed LoRA terms of the CTA's last segment (0: none)
};

template <int N>
struct GemmCfg {
  static constexpr int kBSlot = N * 128;        // activation chunk slot
  static constexpr int kAccCols = N < 16 ? 16 : N;
  static constexpr int kTmemCols = 2 * kAccCols < 32 ? 32 : 2 * kAccCols;  // two accumulators
  static constexpr int kStageTile = 16 * kGemmM * 4;                          // epilogue staging
  static_assert(kBSlot % 1024 == 0, "swizzle atoms must stay 1024-byte aligned");
};

__host__ __device__ inline int gemm_smem_bytes(int ring_bytes, int lora_stage, int lora_delta, int stages) {
  return 1024 + ring_bytes + kGemmGuard + 16 * kGemmM * 4 + lora_stage + lora_delta + (2 * stages + 4) * 8 + 32;
}

template <int N, int KCS>
__global__ void __launch_bounds__(kGemmThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                     const GemmArgs g) {
  using C = GemmCfg<N>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = g.stages;
  const int SB = g.stage_bytes;
  const int AS = g.a_slot;
  uint8_t* tail = smem + S * SB + kGemmGuard;
  float* stile = reinterpret_cast<float*>(tail);  // [16 tokens][128 rows]
  // Rank-16 LoRA epilogue inputs, staged once: down rows rounded to bf16
  // [T][num_slices * 16], then the tokens' adapter ids [T].
  float* lds = reinterpret_cast<float*>(tail + C::kStageTile);
  // The precomputed LoRA terms of the CTA's last segment, [T][128] bf16.
  bf16* sdl = reinterpret_cast<bf16*>(tail + C::kStageTile + g.lora_stage);
  uint64_t* full = reinterpret_cast<uint64_t*>(tail + C::kStageTile + g.lora_stage + g.lora_delta);
  uint64_t* empty = full + S;
  uint64_t* accf = empty + S;  // [2] accumulator ready
  uint64_t* acce = accf + 2;   // [2] accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int32_t* flags = reinterpret_cast<volatile int32_t*>(tmem_slot + 1);  // abort, -, issued, consumed

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int KB = g.kblocks;
  const int64_t band0 = (int64_t)blockIdx.x * g.band_rows;
  // Segments of this band that hold rows (the last band may be short).
  int nseg = g.nseg;
  while (nseg > 0 && band0 + (int64_t)(nseg - 1) * g.seg_rows >= g.e.n_out) --nseg;
  const int n = nseg * KB;  // units

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);  // one arrival per epilogue warp
    }
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
  if (threadIdx.x == 0) PL_TRACE_POINT(0);
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // A TMA instruction costs a fixed issue time however many lanes issue
    // it, so the warp issues up to kGemmIssue units per instruction: lanes
    // 2*KCS*j .. 2*KCS*j + KCS - 1 load unit j's weight chunks (the first
    // one arms the unit's barrier), the next KCS lanes its activation chunks.
    const uint64_t pol = l2_evict_first_policy();
    const int tx = KCS * (g.seg_rows * 128 + C::kBSlot);
    const int pre = g.e.early_weights ? (n < S ? n : S) : 0;
    // Weights are not produced upstream: start the first stages now.
    for (int idx = lane; idx < pre * KCS; idx += 32) {
      const int i = idx / KCS, j = idx % KCS;
      const int seg = i / KB, kb = i % KB;
      if (j == 0) mbar_arrive_expect_tx(&full[i], tx);
      __syncwarp(__activemask());
      tma_load_2d(smem + i * SB + j * AS, &wmap, (kb * KCS + j) * kGemmKC,
                  (int32_t)(band0 + (int64_t)seg * g.seg_rows), &full[i], pol);
    }
    pdl_wait();
    if (lane == 0) PL_TRACE_POINT(1);
    constexpr int kLanesPerUnit = 2 * KCS;
    constexpr int kBatch = 32 / kLanesPerUnit < kGemmIssue ? 32 / kLanesPerUnit : kGemmIssue;
    const int batch = S < kBatch ? S : kBatch;  // a batch never reuses its own stages
    const int jb = lane / kLanesPerUnit, part = lane % kLanesPerUnit;
    const bool is_w = part < KCS;
    const int j = is_w ? part : part - KCS;
    int i0 = 0;
    for (; i0 < n; i0 += batch) {
      const int i = i0 + jb;
      const bool active = jb < batch && i < n;
      const int s = i % S;
      bool ok = true;
      if (active && part == 0 && i >= S) ok = mbar_wait(&empty[s], ((i / S) - 1) & 1);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) set_status(g.e.status, PL_ERR_TIMEOUT);
        flags[0] = 1;
        break;
      }
      __syncwarp();  // every lane of a unit sees its stage free before any copy into it
      const int seg = i / KB, kb = i % KB;
      uint8_t* st = smem + s * SB;
      if (active && part == 0 && i >= pre) mbar_arrive_expect_tx(&full[s], tx);
      __syncwarp();
      if (active) {
        if (is_w) {
          if (i >= pre)
            tma_load_2d(st + j * AS, &wmap, (kb * KCS + j) * kGemmKC, (int32_t)(band0 + (int64_t)seg * g.seg_rows),
                        &full[s], pol);
        } else {
          tma_load_2d(st + KCS * AS + j * C::kBSlot, &xmap, (kb * KCS + j) * kGemmKC, 0, &full[s], 0ull);
        }
      }
    }
    if (lane == 0) flags[2] = i0 < n ? (i0 > pre ? i0 : pre) : n;
    if (lane == 0) PL_TRACE_POINT(9);
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kGemmM, N);
      int i = 0;
      bool ok = true;
      for (; i < n; ++i) {
        const int seg = i / KB, kb = i % KB;
        const int b = seg & 1;
        if (kb == 0 && seg >= 2) ok = mbar_wait(&acce[b], ((seg >> 1) - 1) & 1);
        const int s = i % S;
        if (ok) ok = mbar_wait(&full[s], (i / S) & 1);
        if (!ok) {
          set_status(g.e.status, PL_ERR_TIMEOUT);
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        if (i == 0) PL_TRACE_POINT(2);
        const uint32_t a0 = smem_u32(smem + s * SB);
        const uint32_t b0 = a0 + KCS * AS;
        const uint32_t acc = tmem + (uint32_t)(b * C::kAccCols);
#pragma unroll
        for (int jj = 0; jj < KCS; ++jj) {
#pragma unroll
          for (int k = 0; k < kGemmKC / 16; ++k)
            umma_bf16(acc, umma_desc_k_sw128(a0 + jj * AS + 32 * k), umma_desc_k_sw128(b0 + jj * C::kBSlot + 32 * k),
                      idesc, (kb > 0 || jj > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        if (kb == KB - 1) umma_commit(&accf[b]);
      }
      flags[3] = i;
      PL_TRACE_POINT(3);
      if (!ok) {
        // Release the epilogue for the segments that will not be computed.
        for (int seg = i / KB; seg < nseg; ++seg) umma_commit(&accf[seg & 1]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();  // residual, LoRA down and adapter ids come from upstream kernels
    const int ew = warp - 2;     // epilogue warp 0..3
    const int q = warp & 3;      // TMEM lane quadrant this warp may read
    const int row = 32 * q + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    const int T = g.e.T;
    constexpr int kEpiThreads = 128;
    const int R = g.e.num_slices * 16;
    const float* sdown = nullptr;
    const int32_t* sad = nullptr;
    if (g.lora_stage) {
      int32_t* lad = reinterpret_cast<int32_t*>(lds + T * R);
      for (int idx = ew * 32 + lane; idx < T * R; idx += kEpiThreads)
        lds[idx] = bfr(g.e.lora_down[(int64_t)(idx / R) * g.e.down_stride + idx % R]);
      for (int t2 = ew * 32 + lane; t2 < T; t2 += kEpiThreads)
        lad[t2] = g.e.tok_adapter != nullptr ? g.e.tok_adapter[t2] : 0;
      named_barrier(1, kEpiThreads);
      sdown = lds;
      sad = lad;
    }
    // The LoRA terms of the CTA's last segment, computed while the weights
    // stream: its epilogue, at the very end of the CTA, then only adds them.
    const int seg_pre = (g.lora_delta && nseg > 0) ? nseg - 1 : -1;
    if (seg_pre >= 0) {
      const int64_t row0 = band0 + (int64_t)seg_pre * g.seg_rows;
      int64_t row_end = row0 + g.seg_rows;
      if (row_end > g.e.n_out) row_end = g.e.n_out;
      // lane: rows 4*lane .. 4*lane+3 of the segment; warp ew: a contiguous
      // quarter of the tokens, so a B row set is loaded once per adapter run
      const int64_t o0 = row0 + 4 * lane;
      int sl[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sl[i] = 0;
        while (sl[i] < g.e.num_slices - 1 && o0 + i >= g.e.slice_end[sl[i]]) ++sl[i];
      }
      const bool rows_ok = o0 + 4 <= row_end;
      int cur = -1;
      uint4 b[4][2] = {};
      const int tq = (T + 3) / 4;
      for (int tok = ew * tq; tok < T && tok < (ew + 1) * tq; ++tok) {
        const int ad = sad[tok];
        float dv[4] = {0.f, 0.f, 0.f, 0.f};
        if (ad >= 0 && rows_ok) {
          if (ad != cur) {
            cur = ad;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint4* br = reinterpret_cast<const uint4*>(g.e.lora_b + ((int64_t)ad * g.e.n_out + o0 + i) * 16);
              b[i][0] = br[0];
              b[i][1] = br[1];
            }
          }
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dv[i] = bfr(bfr(lora_dot16(b[i], sdown + tok * R + sl[i] * 16)) * g.e.lora_scale);
        }
        if (rows_ok)
          *reinterpret_cast<uint2*>(sdl + tok * kGemmM + 4 * lane) =
              make_uint2(pack_bf16x2(dv[0], dv[1]), pack_bf16x2(dv[2], dv[3]));
      }
      named_barrier(1, kEpiThreads);
      if (threadIdx.x == 64) PL_TRACE_POINT(10);
    }
    for (int seg = 0; seg < nseg; ++seg) {
      const int b = seg & 1;
      if (!mbar_wait(&accf[b], (seg >> 1) & 1)) {
        set_status(g.e.status, PL_ERR_TIMEOUT);
        flags[0] = 1;
      }
      tc_fence_after();
      if (threadIdx.x == 64) {
        if (seg == 0) PL_TRACE_POINT(4);
        PL_TRACE_MAX(5);
      }
      const int64_t row0 = band0 + (int64_t)seg * g.seg_rows;
      int64_t row_end = row0 + g.seg_rows;
      if (row_end > g.e.n_out) row_end = g.e.n_out;
      const uint32_t acc = lane_base + (uint32_t)(b * C::kAccCols);
      const int64_t o4 = row0 + 4 * lane;
      // Stage [16 tokens][128 rows] through shared memory, then warp ew
      // finishes tokens 4ew .. 4ew+3 of the chunk (4 rows a lane; adjacent
      // tokens usually share an adapter).
#pragma unroll 1
      for (int c = 0; c < N / 16 && 16 * c < T; ++c) {
        float v[16];
        tmem_ld16(acc + 16 * c, v);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) stile[jj * kGemmM + row] = v[jj];
        named_barrier(1, kEpiThreads);
        if (!flags[0] && o4 < row_end) {
          int toks[4];
          float vals[4][4];
          int nt = 0;
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const int jj = 4 * ew + h;
            toks[h] = 16 * c + jj;
            const float4 r4 = *reinterpret_cast<const float4*>(stile + jj * kGemmM + 4 * lane);
            vals[h][0] = r4.x;
            vals[h][1] = r4.y;
            vals[h][2] = r4.z;
            vals[h][3] = r4.w;
            if (16 * c + jj < T) nt = h + 1;
          }
          epilogue_rows4_x4(g.e, o4, toks, nt, vals, sdown, R, sad, seg == seg_pre ? sdl : nullptr, row0,
                            row_end);
        }
        named_barrier(1, kEpiThreads);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);
    }
    if (threadIdx.x == 64) PL_TRACE_POINT(7);
  }

  // ------------------------------------------------------------ teardown
  __syncthreads();
  if (threadIdx.x == 0) {
    // Loads issued but never consumed (abort only) must land before exit.
    const int issued = flags[2], consumed = flags[3];
    for (int i = consumed; i < issued; ++i) (void)mbar_wait(&full[i % S], (i / S) & 1);
  }
  if (lane == 0) PL_TRACE_MAX(8);
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
PL_TRACE_READER(pl_trace_read_gemm)

namespace {

struct MapKey2 {
  const void* ptr;
  int64_t inner, rows, stride;
  int32_t box_rows, kcs, dev;
  bool operator==(const MapKey2& o) const {
    return ptr == o.ptr && inner == o.inner && rows == o.rows && stride == o.stride && box_rows == o.box_rows &&
           kcs == o.kcs && dev == o.dev;
  }
};
constexpr int kMap2Cache = 512;
struct Map2Cache {
  std::mutex mu;
  MapKey2 key[kMap2Cache];
  CUtensorMap map[kMap2Cache];
  int used = 0, next = 0;
};
Map2Cache g_map2;

// bf16 matrix [rows][inner] with a row stride of `stride` elements, read in
// tiles of box_rows x (kcs x 64) with 128-byte swizzling; out-of-range rows
// and chunks read as zero.  kcs == 1: 2-D map (inner, rows).  kcs > 1
// (inner % 64 == 0): 3-D map (64, rows, inner / 64) whose chunk dimension
// steps 128 bytes along the row, so one copy lands kcs consecutive
// [box_rows][64] swizzled tiles.
int32_t matrix_map(const void* ptr, int64_t inner, int64_t rows, int64_t stride, int box_rows, int kcs,
                   CUtensorMap* out) {
  int dev = 0;
  cudaGetDevice(&dev);
  MapKey2 k{ptr, inner, rows, stride, box_rows, kcs, dev};
  std::lock_guard<std::mutex> lock(g_map2.mu);
  for (int i = 0; i < g_map2.used; ++i)
    if (g_map2.key[i] == k) {
      *out = g_map2.map[i];
      return PL_OK;
    }
  pl_host::EncodeTiledFn enc = pl_host::encode_tiled_fn();
  if (enc == nullptr) return PL_ERR_CUDA;
  CUtensorMap m;
  CUresult r;
  if (kcs == 1) {
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
    cuuint32_t box[2] = {(cuuint32_t)pl::kGemmKC, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[3] = {(cuuint64_t)pl::kGemmKC, (cuuint64_t)rows, (cuuint64_t)(inner / pl::kGemmKC)};
    cuuint64_t strides[2] = {(cuuint64_t)stride * 2, (cuuint64_t)pl::kGemmKC * 2};
    cuuint32_t box[3] = {(cuuint32_t)pl::kGemmKC, (cuuint32_t)box_rows, (cuuint32_t)kcs};
    cuuint32_t estr[3] = {1, 1, 1};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return PL_ERR_UNSUPPORTED;
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

constexpr int kGemmRingBudget = 176 * 1024;
constexpr int kLoraStageMax = 16 * 1024;

int gemm_smem_optin() {
  static int limit[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 227 * 1024;
  if (limit[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0)
      v = 227 * 1024;
    limit[dev] = v;
  }
  return limit[dev];
}

struct GemmShape {
  int n, kcs, seg_rows, nseg, band_rows, kblocks, ctas, a_slot, stage_bytes, stages;
};

// Row bands: the fewest rows per CTA (a multiple of 4) that cover n_out
// with at most max_ctas CTAs, cut into nseg equal segments of <= 128 rows.
// K blocks of kcs x 64 columns (kcs 4 up to 32 tokens, 2 at 64, 1 at 128:
// a stage stays small enough for several of them); as many ring stages as
// fit.
GemmShape gemm_shape(int tokens, int k_in, int n_out, int max_ctas) {
  GemmShape s;
  s.n = gemm_n(tokens);
  s.kcs = s.n <= 32 ? 4 : (s.n == 64 ? 2 : 1);
  const int per = (int)(((int64_t)n_out + max_ctas - 1) / max_ctas);
  s.nseg = (per + pl::kGemmM - 1) / pl::kGemmM;
  const int seg = (int)(((int64_t)n_out + (int64_t)max_ctas * s.nseg - 1) / ((int64_t)max_ctas * s.nseg));
  s.seg_rows = (seg + 3) & ~3;
  if (s.seg_rows > pl::kGemmM) s.seg_rows = pl::kGemmM;
  s.band_rows = s.seg_rows * s.nseg;
  s.ctas = (int)(((int64_t)n_out + s.band_rows - 1) / s.band_rows);
  const int block_cols = pl::kGemmKC * s.kcs;
  s.kblocks = (k_in + block_cols - 1) / block_cols;
  s.a_slot = ((s.seg_rows + 7) & ~7) * 128;
  s.stage_bytes = s.kcs * (s.a_slot + s.n * 128);
  int stages = kGemmRingBudget / s.stage_bytes;
  if (stages > 8) stages = 8;
  s.stages = stages < 2 ? 2 : stages;
  return s;
}

template <int N, int KCS>
int32_t launch_gemm(const CUtensorMap& wm, const CUtensorMap& xm, const pl::GemmArgs& g, int ctas, void* stream) {
  auto kern = pl::linear_tc_kernel<N, KCS>;
  const int smem = pl::gemm_smem_bytes(g.stages * g.stage_bytes, g.lora_stage, g.lora_delta, g.stages);
  int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  if (st != PL_OK) return st;
  return pl_host::launch_pdl(kern, dim3(ctas), dim3(pl::kGemmThreads), smem, stream, wm, xm, g);
}

template <int N>
int32_t launch_gemm_n(int kcs, const CUtensorMap& wm, const CUtensorMap& xm, const pl::GemmArgs& g, int ctas,
                      void* stream) {
  (void)kcs;  // fixed by N, as in gemm_shape
  if constexpr (N == 128) return launch_gemm<N, 1>(wm, xm, g, ctas, stream);
  else if constexpr (N == 64) return launch_gemm<N, 2>(wm, xm, g, ctas, stream);
  else return launch_gemm<N, 4>(wm, xm, g, ctas, stream);
}

int sm_count_or_default() {
  const int sms = pl_host::sm_count();
  return sms > 0 ? sms : 148;
}

}  // namespace

extern "C" int32_t pl_linear_gemm_plan(int32_t num_tokens, int32_t k_in, int32_t n_out, int32_t num_ctas,
                                       pl_gemm_plan_t* plan) {
  if (plan == nullptr || num_tokens < 1 || num_tokens > 128 || k_in <= 0 || n_out <= 0 || num_ctas < 0)
    return PL_ERR_INVALID_ARGUMENT;
  const GemmShape s = gemm_shape(num_tokens, k_in, n_out, num_ctas > 0 ? num_ctas : sm_count_or_default());
  plan->ctas = s.ctas;
  plan->max_slots = 1;
  plan->workspace_bytes = 0;
  return PL_OK;
}

extern "C" int32_t pl_linear_lora_gemm(const void* x, int64_t x_stride, int32_t num_tokens, int32_t k_in,
                                       const void* w, int32_t n_out, const void* bias, const float* lora_down,
                                       int64_t down_stride, const void* lora_b, int32_t lora_rank, float lora_scale,
                                       const int32_t* slice_end, int32_t num_slices, const int32_t* tok_adapter,
                                       const void* residual, int64_t res_stride, void* y, int64_t y_stride,
                                       int32_t num_ctas, void* workspace, int64_t workspace_bytes, int32_t flags,
                                       int32_t* status_dev, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (num_tokens == 0 || n_out == 0) return PL_OK;
  if (x == nullptr || w == nullptr || y == nullptr || num_tokens < 0 || num_tokens > 128 || k_in <= 0 ||
      n_out < 0 || num_ctas < 0)
    return PL_ERR_INVALID_ARGUMENT;
  if (k_in % 8 != 0 || x_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15))
    return PL_ERR_UNSUPPORTED;
  if (lora_b != nullptr && (lora_down == nullptr || lora_rank <= 0 || num_slices < 1 || num_slices > 4 ||
                            (num_slices > 1 && slice_end == nullptr)))
    return PL_ERR_INVALID_ARGUMENT;
  const GemmShape sh = gemm_shape(num_tokens, k_in, n_out, num_ctas > 0 ? num_ctas : sm_count_or_default());
  CUtensorMap wm, xm;
  int32_t st = matrix_map(w, k_in, n_out, k_in, sh.seg_rows, 1, &wm);
  if (st == PL_OK) st = matrix_map(x, k_in, num_tokens, x_stride, sh.n, 1, &xm);
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
  g.kblocks = sh.kblocks;
  g.band_rows = sh.band_rows;
  g.seg_rows = sh.seg_rows;
  g.nseg = sh.nseg;
  g.a_slot = sh.a_slot;
  g.stage_bytes = sh.stage_bytes;
  g.stages = sh.stages;
  // Rank-16 LoRA: stage the (small) down rows and adapter ids in shared
  // memory so the epilogue reads them once per CTA instead of per element,
  // and compute the last segment's LoRA terms ahead when they fit.
  if (lora_b != nullptr && lora_rank == 16 && (reinterpret_cast<uintptr_t>(lora_b) & 15) == 0) {
    const int64_t bytes = (int64_t)num_tokens * a.num_slices * 16 * 4 + (((int64_t)num_tokens * 4 + 15) & ~int64_t(15));
    if (bytes <= kLoraStageMax) g.lora_stage = static_cast<int32_t>(bytes);
    const int32_t delta = num_tokens * pl::kGemmM * 2;
    if (g.lora_stage &&
        pl::gemm_smem_bytes(sh.stages * sh.stage_bytes, g.lora_stage, delta, sh.stages) <= gemm_smem_optin())
      g.lora_delta = delta;
  }

  switch (sh.n) {
    case 16: return launch_gemm_n<16>(sh.kcs, wm, xm, g, sh.ctas, stream);
    case 32: return launch_gemm_n<32>(sh.kcs, wm, xm, g, sh.ctas, stream);
    case 64: return launch_gemm_n<64>(sh.kcs, wm, xm, g, sh.ctas, stream);
    default: return launch_gemm_n<128>(sh.kcs, wm, xm, g, sh.ctas, stream);
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
