// Multi-token LoRA linear (batched decode and prefill chunks, 1..128 tokens)
// on the 5th-generation tensor cores, plus the small activation kernels that
// feed it.
//
// pl_linear_lora_gemm computes y[t, n] = epilogue(sum_k x[t, k] * w[n, k]).
// Work is cut into units of one 128-row weight tile x one K block (4 chunks
// of 64 columns, 2 when N = 128); the persistent grid has one CTA per SM and
// CTA c takes the contiguous unit range [c*U/P, (c+1)*U/P) -- every SM
// streams the same number of bytes whatever the tile count (per-SM copy
// throughput, not HBM, is the limit when SMs idle).  Per CTA:
//   warp 0     streams each unit's weight tile (128 rows x 256 columns, one
//              3-D TMA copy reading 512 contiguous bytes per row) and the
//              activation tile into a shared-memory ring, several units per
//              issuing instruction;
//   warp 1     (one lane) issues tcgen05.mma (M = 128, N = tokens padded to
//              16/32/64/128, K = 16) into one of two tensor-memory
//              accumulators, one per tile segment;
//   warps 2-5  read a finished accumulator with tcgen05.ld (warp w owns
//              lanes 32(w%4)..) while the next segment accumulates, and run
//              the decode GEMV's epilogue (bias, per-token LoRA expand with
//              the token's adapter, residual; the reference's bf16 rounding
//              points), staged through shared memory into 8-byte stores.
// A tile split between CTAs is finished by the last contributor (arrival
// ticket per tile), which adds the contributors' fp32 partials in CTA order
// -- deterministic -- and runs the epilogue.  No wait depends on another CTA.
#include "pl_linear_common.cuh"

#include <mutex>

namespace pl {

constexpr int kGemmM = 128;      // weight rows per tile (UMMA M)
constexpr int kGemmKC = 64;      // K per chunk: one 128-byte swizzled row of bf16
constexpr int kGemmThreads = 192;
constexpr int kGemmIssue = 4;    // units per producer TMA instruction

struct GemmArgs {
  GemvArgs e;          // epilogue fields: n_out, bias, LoRA, residual, y, status; T, K
  int32_t kblocks;     // K blocks per tile
  int32_t units;       // m_tiles * kblocks
  int32_t stages;
  int32_t max_slots;   // partial slots per tile
  float* partial;      // [m_tiles][max_slots][N][128] fp32
  int32_t* counters;   // [m_tiles] arrival tickets, zero between calls
  int32_t lora_stage;  // bytes of shared memory holding the rank-16 LoRA down rows and adapter ids (0: none)
  int32_t lora_delta;  // bytes holding the precomputed LoRA terms of the CTA's last tile (0: none)
};

// N: tokens padded (UMMA N).  KCS: 64-column chunks per K block; with KCS > 1
// the tiles come from 3-D tensor maps (64, rows, K / 64) so that one copy
// reads KCS x 128 contiguous bytes of every weight row.
template <int N, int KCS>
struct GemmCfg {
  static constexpr int kATile = kGemmM * 128;   // 16 KB weight tile per chunk
  static constexpr int kBTile = N * 128;        // activation tile per chunk
  static constexpr int kABytes = KCS * kATile;
  static constexpr int kBBytes = KCS * kBTile;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kAccCols = N < 16 ? 16 : N;
  static constexpr int kTmemCols = 2 * kAccCols < 32 ? 32 : 2 * kAccCols;  // two accumulators
  static constexpr int kStageTile = 16 * kGemmM * 4;                          // epilogue staging
  static_assert(kBTile % 1024 == 0, "swizzle atoms must stay 1024-byte aligned");
};

__host__ __device__ inline int gemm_smem_bytes(int stage_bytes, int stages, int lora_stage) {
  return 1024 + stages * stage_bytes + 16 * kGemmM * 4 + lora_stage + (2 * stages + 4) * 8 + 32;
}
__host__ __device__ inline int gemm_smem_bytes(int stage_bytes, int stages, int lora_stage, int lora_delta) {
  return gemm_smem_bytes(stage_bytes, stages, lora_stage) + lora_delta;
}

__host__ __device__ inline int unit_begin(int c, int units, int ctas) {
  return (int)(((int64_t)c * units) / ctas);
}
// The CTA whose unit range holds unit u.
__host__ __device__ inline int cta_of_unit(int u, int units, int ctas) {
  int c = (int)(((int64_t)u * ctas) / units);
  while (c + 1 < ctas && unit_begin(c + 1, units, ctas) <= u) ++c;
  while (c > 0 && unit_begin(c, units, ctas) > u) --c;
  return c;
}

template <int KCS>
__device__ __forceinline__ void gemm_tile_load(void* dst, const CUtensorMap* map, int kb, int row0, uint64_t* bar,
                                               uint64_t pol) {
  if constexpr (KCS == 1)
    tma_load_2d(dst, map, kb * kGemmKC, row0, bar, pol);
  else
    tma_load_3d(dst, map, 0, row0, kb * KCS, bar, pol);
}

template <int N, int KCS>
__global__ void __launch_bounds__(kGemmThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                     const GemmArgs g) {
  using C = GemmCfg<N, KCS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = g.stages;
  float* stile = reinterpret_cast<float*>(smem + S * C::kStageBytes);  // [16 tokens][128 rows]
  // Rank-16 LoRA epilogue inputs, staged once: down rows rounded to bf16
  // [T][num_slices * 16], then the tokens' adapter ids [T].
  float* lds = reinterpret_cast<float*>(smem + S * C::kStageBytes + C::kStageTile);
  // The precomputed LoRA terms of the CTA's last tile, [T][128] bf16.
  bf16* sdl = reinterpret_cast<bf16*>(smem + S * C::kStageBytes + C::kStageTile + g.lora_stage);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * C::kStageBytes + C::kStageTile + g.lora_stage +
                                               g.lora_delta);
  uint64_t* empty = full + S;
  uint64_t* accf = empty + S;  // [2] accumulator ready
  uint64_t* acce = accf + 2;   // [2] accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int32_t* flags = reinterpret_cast<volatile int32_t*>(tmem_slot + 1);  // abort, last, issued, consumed

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int P = gridDim.x, U = g.units, KB = g.kblocks;
  const int u0 = unit_begin(blockIdx.x, U, P), u1 = unit_begin(blockIdx.x + 1, U, P);
  const int n = u1 - u0;  // >= 1: the grid never exceeds the unit count

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
    // it, so the warp issues up to kGemmIssue units per instruction: lane 2j
    // loads unit j's weight tile (and arms its barrier), lane 2j+1 its
    // activation tile.
    const uint64_t pol = l2_evict_first_policy();
    const int pre = g.e.early_weights ? (n < S ? n : S) : 0;
    for (int i = lane; i < pre; i += 32) {  // weights are not produced upstream: start them now
      const int u = u0 + i;
      mbar_arrive_expect_tx(&full[i], C::kStageBytes);
      gemm_tile_load<KCS>(smem + i * C::kStageBytes, &wmap, u % KB, (u / KB) * kGemmM, &full[i], pol);
    }
    pdl_wait();
    if (lane == 0) PL_TRACE_POINT(1);
    const int jb = lane >> 1, kind = lane & 1;
    // A batch of units is issued only once all of their stages are free, so
    // it stays smaller than the ring: a batch as deep as the ring would drain
    // it before every refill and leave the CTA idle for a whole memory
    // latency per ring's worth of data.
    int batch = S - 1 < kGemmIssue ? S - 1 : kGemmIssue;
    if (batch < 1) batch = 1;
    int i0 = 0;
    for (; i0 < n; i0 += batch) {
      const int i = i0 + jb;
      const bool active = lane < 2 * batch && i < n;
      const int s = i % S;
      bool ok = true;
      if (active && i >= S) ok = mbar_wait(&empty[s], ((i / S) - 1) & 1);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) set_status(g.e.status, PL_ERR_TIMEOUT);
        flags[0] = 1;
        break;
      }
      const int u = u0 + i;
      uint8_t* st = smem + s * C::kStageBytes;
      if (active && kind == 0 && i >= pre) mbar_arrive_expect_tx(&full[s], C::kStageBytes);
      __syncwarp();
      if (active) {
        if (kind == 0) {
          if (i >= pre) gemm_tile_load<KCS>(st, &wmap, u % KB, (u / KB) * kGemmM, &full[s], pol);
        } else {
          gemm_tile_load<KCS>(st + C::kABytes, &xmap, u % KB, 0, &full[s], 0ull);
        }
      }
    }
    if (lane == 0) flags[2] = i0 < n ? (i0 > pre ? i0 : pre) : n;
    if (lane == 0) PL_TRACE_POINT(9);
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kGemmM, N);
      int i = 0, seg = 0;
      bool ok = true;
      for (; i < n; ++i) {
        const int u = u0 + i, kb = u % KB;
        const bool first = (i == 0 || kb == 0), last = (i == n - 1 || kb == KB - 1);
        const int b = seg & 1;
        if (first && seg >= 2) ok = mbar_wait(&acce[b], ((seg >> 1) - 1) & 1);
        const int s = i % S;
        if (ok) ok = mbar_wait(&full[s], (i / S) & 1);
        if (!ok) {
          set_status(g.e.status, PL_ERR_TIMEOUT);
          flags[0] = 1;
          break;
        }
        tc_fence_after();
        if (i == 0) PL_TRACE_POINT(2);
        const uint32_t a0 = smem_u32(smem + s * C::kStageBytes);
        const uint32_t b0 = a0 + C::kABytes;
        const uint32_t acc = tmem + (uint32_t)(b * C::kAccCols);
#pragma unroll
        for (int j = 0; j < KCS; ++j) {
#pragma unroll
          for (int k = 0; k < kGemmKC / 16; ++k)
            umma_bf16(acc, umma_desc_k_sw128(a0 + j * C::kATile + 32 * k),
                      umma_desc_k_sw128(b0 + j * C::kBTile + 32 * k), idesc, (!first || j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        if (last) {
          umma_commit(&accf[b]);
          ++seg;
        }
      }
      flags[3] = i;
      PL_TRACE_POINT(3);
      if (!ok) {
        // Release the epilogue for the segments that will not be computed.
        for (int i2 = i; i2 < n; ++i2) {
          const int kb = (u0 + i2) % KB;
          if (i2 == n - 1 || kb == KB - 1) {
            umma_commit(&accf[seg & 1]);
            ++seg;
          }
        }
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
    // The LoRA terms of the tile that this CTA's last segment covers: its
    // epilogue (a whole tile, or the merge of the shared tile's partials, at
    // the very end of the CTA) then only adds them.  Computed here, while the
    // first accumulator is still being filled.
    // Only a CTA with at least half a tile of units of its own: with fewer,
    // a tile has many contributors that finish together, the precomputed terms
    // are mostly unused, and computing them delays the partials.
    const int t_pre = (g.lora_delta && 2 * n >= KB) ? (u1 - 1) / KB : -1;
    if (t_pre >= 0) {
      const int64_t row0 = (int64_t)t_pre * kGemmM;
      // lane: rows 4*lane .. 4*lane+3 of the tile; warp ew: a contiguous quarter
      // of the tokens, so a B row set is loaded once per adapter run
      const int64_t o0 = row0 + 4 * lane;
      int sl[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sl[i] = 0;
        while (sl[i] < g.e.num_slices - 1 && o0 + i >= g.e.slice_end[sl[i]]) ++sl[i];
      }
      const bool rows_ok = o0 + 4 <= g.e.n_out;
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
        *reinterpret_cast<uint2*>(sdl + tok * kGemmM + 4 * lane) =
            make_uint2(pack_bf16x2(dv[0], dv[1]), pack_bf16x2(dv[2], dv[3]));
      }
      named_barrier(1, kEpiThreads);
    }
    int seg = 0;
    for (int i = 0; i < n;) {
      const int u = u0 + i, t = u / KB, ka = u % KB;
      int len = KB - ka;
      if (len > n - i) len = n - i;
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
      const uint32_t acc = lane_base + (uint32_t)(b * C::kAccCols);
      const int64_t o4 = (int64_t)t * kGemmM + 4 * lane;
      const bool whole = (ka == 0 && len == KB);
      if (whole) {
        // The whole tile is here: stage [16 tokens][128 rows] through shared
        // memory, then warp ew finishes tokens ew, ew+4, ... (4 rows a lane).
#pragma unroll 1
        for (int c = 0; c < N / 16 && 16 * c < T; ++c) {
          float v[16];
          tmem_ld16(acc + 16 * c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) stile[j * kGemmM + row] = v[j];
          named_barrier(1, kEpiThreads);
          if (!flags[0]) {
            // tokens 4ew .. 4ew+3 of this chunk (adjacent tokens usually
            // share an adapter), finished together
            int toks[4];
            float vals[4][4];
            int nt = 0;
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const int j = 4 * ew + h;
              toks[h] = 16 * c + j;
              const float4 r4 = *reinterpret_cast<const float4*>(stile + j * kGemmM + 4 * lane);
              vals[h][0] = r4.x;
              vals[h][1] = r4.y;
              vals[h][2] = r4.z;
              vals[h][3] = r4.w;
              if (16 * c + j < T) nt = h + 1;
            }
            if (g.e.silu_pairs)
              epilogue_silu_pairs(g.e, t, lane, toks, nt, vals);
            else
              epilogue_rows4_x4(g.e, o4, toks, nt, vals, sdown, R, sad, t == t_pre ? sdl : nullptr,
                                (int64_t)t * kGemmM);
          }
          named_barrier(1, kEpiThreads);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[b]);
      } else {
        // Part of a tile: leave the fp32 partial in this CTA's slot; the last
        // contributor adds the slots in order and runs the epilogue.
        const int c_first = cta_of_unit(t * KB, U, P);
        const int c_last = cta_of_unit(t * KB + KB - 1, U, P);
        const int slot = blockIdx.x - c_first;
        float* mine = g.partial + ((int64_t)t * g.max_slots + slot) * N * kGemmM;
#pragma unroll 1
        for (int c = 0; c < N / 16 && 16 * c < T; ++c) {
          float v[16];
          tmem_ld16(acc + 16 * c, v);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (16 * c + j < T) __stcg(mine + (16 * c + j) * kGemmM + row, v[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[b]);
        __threadfence();
        named_barrier(1, kEpiThreads);
        if (ew == 0 && lane == 0) {
          const int32_t ticket = atomicAdd(&g.counters[t], 1);
          flags[1] = ticket == c_last - c_first ? 1 : 0;
        }
        named_barrier(1, kEpiThreads);
        if (threadIdx.x == 64) PL_TRACE_MAX(6);
        if (flags[1]) {
          __threadfence();
          const int nslots = c_last - c_first + 1;
          const float* base = g.partial + (int64_t)t * g.max_slots * N * kGemmM + 4 * lane;
          // Four tokens x four slots of loads in flight per lane; slots are
          // added in order, so the sum does not depend on timing.
#pragma unroll 1
          for (int tok = 4 * ew; tok < T; tok += 16) {
            float a4[4][4] = {};
            int toks[4];
            int nt = 0;
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              toks[h] = tok + h;
              if (tok + h < T) nt = h + 1;
            }
#pragma unroll 1
            for (int sl = 0; sl < nslots; sl += 4) {
              float4 p[4][4];
#pragma unroll
              for (int h = 0; h < 4; ++h)
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  p[h][k] = (sl + k < nslots && h < nt)
                                ? __ldcg(reinterpret_cast<const float4*>(
                                      base + ((int64_t)(sl + k) * N + tok + h) * kGemmM))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
              for (int h = 0; h < 4; ++h)
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  a4[h][0] += p[h][k].x;
                  a4[h][1] += p[h][k].y;
                  a4[h][2] += p[h][k].z;
                  a4[h][3] += p[h][k].w;
                }
            }
            if (!flags[0]) {
              if (g.e.silu_pairs)
                epilogue_silu_pairs(g.e, t, lane, toks, nt, a4);
              else
                epilogue_rows4_x4(g.e, o4, toks, nt, a4, sdown, R, sad, t == t_pre ? sdl : nullptr,
                                  (int64_t)t * kGemmM);
            }
          }
          if (ew == 0 && lane == 0) g.counters[t] = 0;
        }
        named_barrier(1, kEpiThreads);  // flags[1] is reused by the next segment
      }
      i += len;
      ++seg;
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

int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

constexpr int kGemmSmemBudget = 200 * 1024;
constexpr int kLoraStageMax = 16 * 1024;
// Dynamic shared memory a CTA may opt into on the current device (227 KB on
// B200), read once per device.
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
  int n, kcs, stages, m_tiles, kblocks, units, ctas, max_slots, stage_bytes;
};

// Tile geometry: K blocks of kcs x 64 columns (kcs 4, or 2 at N = 128, when
// K % 64 == 0; else 1), as many ring stages as fit; `ctas` CTAs (one per SM
// by default) share the m_tiles x kblocks units evenly.
GemmShape gemm_shape(int tokens, int k_in, int n_out, int ctas, bool allow_3d) {
  GemmShape s;
  s.n = gemm_n(tokens);
  s.kcs = (allow_3d && k_in % pl::kGemmKC == 0) ? (s.n == 128 ? 2 : 4) : 1;
  s.stage_bytes = s.kcs * (pl::kGemmM * 128 + s.n * 128);
  s.m_tiles = (n_out + pl::kGemmM - 1) / pl::kGemmM;
  const int block_cols = pl::kGemmKC * s.kcs;
  s.kblocks = (k_in + block_cols - 1) / block_cols;
  s.units = s.m_tiles * s.kblocks;
  s.ctas = ctas < s.units ? ctas : s.units;
  int stages = kGemmSmemBudget / s.stage_bytes;
  if (stages > 8) stages = 8;
  s.stages = stages < 2 ? 2 : stages;
  s.max_slots = 1;
  for (int t = 0; t < s.m_tiles; ++t) {
    const int c0 = pl::cta_of_unit(t * s.kblocks, s.units, s.ctas);
    const int c1 = pl::cta_of_unit(t * s.kblocks + s.kblocks - 1, s.units, s.ctas);
    if (c1 - c0 + 1 > s.max_slots) s.max_slots = c1 - c0 + 1;
  }
  return s;
}

int64_t gemm_workspace_bytes(const GemmShape& s) {
  int64_t b = align256((int64_t)s.m_tiles * 4);
  if (s.max_slots > 1) b += (int64_t)s.m_tiles * s.max_slots * s.n * pl::kGemmM * 4;
  return b;
}

// Shared-memory bytes of the rank-16 LoRA staging (down rows + adapter ids)
// and of the precomputed last-tile LoRA terms, 0 when a part is not used.
void gemm_lora_smem(int tokens, int num_slices, int lora_rank, bool b_aligned, const GemmShape& sh, int32_t* stage,
                    int32_t* delta) {
  *stage = *delta = 0;
  if (lora_rank != 16 || !b_aligned) return;
  const int64_t bytes = (int64_t)tokens * num_slices * 16 * 4 + (((int64_t)tokens * 4 + 15) & ~int64_t(15));
  if (bytes > kLoraStageMax) return;
  *stage = static_cast<int32_t>(bytes);
  const int32_t d = tokens * pl::kGemmM * 2;  // when it fits beside the ring
  if (pl::gemm_smem_bytes(sh.stage_bytes, sh.stages, *stage, d) <= gemm_smem_optin()) *delta = d;
}

template <int N, int KCS>
int32_t launch_gemm(const CUtensorMap& wm, const CUtensorMap& xm, const pl::GemmArgs& g, int ctas, int stages,
                    void* stream) {
  auto kern = pl::linear_tc_kernel<N, KCS>;
  const int smem = pl::gemm_smem_bytes(pl::GemmCfg<N, KCS>::kStageBytes, stages, g.lora_stage, g.lora_delta);
  int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(kern), smem);
  if (st != PL_OK) return st;
  return pl_host::launch_pdl(kern, dim3(ctas), dim3(pl::kGemmThreads), smem, stream, wm, xm, g);
}

template <int N>
int32_t launch_gemm_n(int kcs, const CUtensorMap& wm, const CUtensorMap& xm, const pl::GemmArgs& g, int ctas,
                      int stages, void* stream) {
  if (kcs == 1) return launch_gemm<N, 1>(wm, xm, g, ctas, stages, stream);
  if constexpr (N == 128) return launch_gemm<N, 2>(wm, xm, g, ctas, stages, stream);
  else return launch_gemm<N, 4>(wm, xm, g, ctas, stages, stream);
}

int sm_count_or_default() {
  const int sms = pl_host::sm_count();
  return sms > 0 ? sms : 148;
}

// One CTA per SM when the row tiles alone cover the device; otherwise 7/8 of
// the SMs, which measured faster (fewer contributors per shared tile, less
// partial traffic) on the 4096-row projections.
int default_ctas(int n_out) {
  const int sms = sm_count_or_default();
  const int m_tiles = (n_out + pl::kGemmM - 1) / pl::kGemmM;
  return m_tiles >= sms ? sms : (sms * 7) / 8;
}

}  // namespace

extern "C" int32_t pl_linear_gemm_plan(int32_t num_tokens, int32_t k_in, int32_t n_out, int32_t num_ctas,
                                       pl_gemm_plan_t* plan) {
  if (plan == nullptr || num_tokens < 1 || num_tokens > 128 || k_in <= 0 || n_out <= 0 || num_ctas < 0)
    return PL_ERR_INVALID_ARGUMENT;
  const GemmShape s = gemm_shape(num_tokens, k_in, n_out, num_ctas > 0 ? num_ctas : default_ctas(n_out),
                                 k_in % pl::kGemmKC == 0);
  plan->ctas = s.ctas;
  plan->max_slots = s.max_slots;
  plan->workspace_bytes = gemm_workspace_bytes(s);
  return PL_OK;
}

extern "C" int32_t pl_linear_gemm_lora_precompute(int32_t num_tokens, int32_t k_in, int32_t n_out, int32_t num_ctas,
                                                  int32_t lora_rank, int32_t num_slices) {
  if (num_tokens < 1 || num_tokens > 128 || k_in <= 0 || n_out <= 0 || num_ctas < 0 || num_slices < 1 ||
      num_slices > 4)
    return PL_ERR_INVALID_ARGUMENT;
  const GemmShape s = gemm_shape(num_tokens, k_in, n_out, num_ctas > 0 ? num_ctas : default_ctas(n_out),
                                 k_in % pl::kGemmKC == 0);
  int32_t stage = 0, delta = 0;
  gemm_lora_smem(num_tokens, num_slices, lora_rank, true, s, &stage, &delta);
  return delta > 0 ? 1 : 0;
}

extern "C" int32_t pl_linear_lora_gemm(const void* x, int64_t x_stride, int32_t num_tokens, int32_t k_in,
                                       const void* w, int32_t n_out, const void* bias, const float* lora_down,
                                       int64_t down_stride, const void* lora_b, int32_t lora_rank, float lora_scale,
                                       const int32_t* slice_end, int32_t num_slices, const int32_t* tok_adapter,
                                       const void* residual, int64_t res_stride, void* y, int64_t y_stride,
                                       int32_t num_ctas, void* workspace, int64_t workspace_bytes, int32_t flags,
                                       int32_t* status_dev, void* stream) {
  if (num_tokens == 0 || n_out == 0) return PL_OK;
  if (x == nullptr || w == nullptr || y == nullptr || num_tokens < 0 || num_tokens > 128 || k_in <= 0 ||
      n_out < 0 || workspace == nullptr || num_ctas < 0)
    return PL_ERR_INVALID_ARGUMENT;
  if (k_in % 8 != 0 || x_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15))
    return PL_ERR_UNSUPPORTED;
  if (lora_b != nullptr && (lora_down == nullptr || lora_rank <= 0 || num_slices < 1 || num_slices > 4 ||
                            (num_slices > 1 && slice_end == nullptr)))
    return PL_ERR_INVALID_ARGUMENT;
  const int ctas = num_ctas > 0 ? num_ctas : default_ctas(n_out);
  GemmShape sh = gemm_shape(num_tokens, k_in, n_out, ctas, true);
  CUtensorMap wm, xm;
  int32_t st = matrix_map(w, k_in, n_out, k_in, pl::kGemmM, sh.kcs, &wm);
  if (st == PL_OK) st = matrix_map(x, k_in, num_tokens, x_stride, sh.n, sh.kcs, &xm);
  if (st == PL_ERR_UNSUPPORTED && sh.kcs > 1) {  // no 3-D map: one chunk per K block
    sh = gemm_shape(num_tokens, k_in, n_out, ctas, false);
    st = matrix_map(w, k_in, n_out, k_in, pl::kGemmM, 1, &wm);
    if (st == PL_OK) st = matrix_map(x, k_in, num_tokens, x_stride, sh.n, 1, &xm);
  }
  if (st != PL_OK) return st;
  if (workspace_bytes < gemm_workspace_bytes(sh) || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return PL_ERR_WORKSPACE_TOO_SMALL;

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
  if (flags & PL_FLAG_SILU_PAIRS) {
    // y gets n_out / 2 columns: 64 per tile, 8-byte stores
    if (lora_b != nullptr || residual != nullptr || bias != nullptr) return PL_ERR_UNSUPPORTED;
    if (n_out % pl::kGemmM != 0 || y_stride % 4 != 0 || (reinterpret_cast<uintptr_t>(y) & 7))
      return PL_ERR_INVALID_ARGUMENT;
    a.silu_pairs = 1;
  }
  a.status = status_dev;
  g.kblocks = sh.kblocks;
  g.units = sh.units;
  g.stages = sh.stages;
  g.max_slots = sh.max_slots;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  g.counters = reinterpret_cast<int32_t*>(ws);
  g.partial = sh.max_slots > 1 ? reinterpret_cast<float*>(ws + align256((int64_t)sh.m_tiles * 4)) : nullptr;
  // Rank-16 LoRA: stage the (small) down rows and adapter ids in shared
  // memory so the epilogue reads them once per CTA instead of per element.
  if (lora_b != nullptr)
    gemm_lora_smem(num_tokens, a.num_slices, lora_rank, (reinterpret_cast<uintptr_t>(lora_b) & 15) == 0, sh,
                   &g.lora_stage, &g.lora_delta);

  switch (sh.n) {
    case 16: return launch_gemm_n<16>(sh.kcs, wm, xm, g, sh.ctas, sh.stages, stream);
    case 32: return launch_gemm_n<32>(sh.kcs, wm, xm, g, sh.ctas, sh.stages, stream);
    case 64: return launch_gemm_n<64>(sh.kcs, wm, xm, g, sh.ctas, sh.stages, stream);
    default: return launch_gemm_n<128>(sh.kcs, wm, xm, g, sh.ctas, sh.stages, stream);
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
