// LoRA linear path for decode (num_tokens <= 8) on sm_100a.
//
// pl_linear_lora_expand_fused streams the weight matrix exactly once: the
// CTA-persistent grid (one CTA per SM) gives each CTA a contiguous range of
// output rows; a producer warp streams 16-row x 512-column tiles of those
// rows into a 5-deep shared-memory ring with 1-D TMA bulk copies (one row
// segment per lane, L2 evict-first), and four consumer warps multiply them
// against the (RMS-normalised / SiLU-gated) activations with mma.sync
// m16n8k16 (weight rows = M, tokens = N, fp32 accumulate).  The epilogue
// adds bias, the LoRA expand (B . down, scale folded into B) and the
// residual with the same bf16 rounding points as the reference's torch ops.
// Rows past n_out come from a second matrix (the LoRA A of the packed
// q/k/v shrink), so the shrink rides along the base projection for free.
//
// pl_lora_shrink_seg and pl_lora_merge_weight are small bandwidth kernels.
#include "pl_linear_common.cuh"

namespace pl {

struct GemvSmem {
  // offsets from a 128-aligned base
  int row_bytes, stage_bytes, nbuf, x_off, zero_off, acc_off, cnt_off, bar_off, misc_off, down_off, total;
};

// down_floats: fp32 LoRA down values the kernel computes itself (T * rank
// with a LoRA A stack in the arguments, else 0).
__host__ __device__ inline GemvSmem gemv_smem_layout(int T, int K, int stages, int kc, int down_floats) {
  GemvSmem L;
  L.row_bytes = kc * 2 + 16;  // padded rows: conflict-free ldmatrix
  L.stage_bytes = kTileRows * L.row_bytes;
  L.nbuf = stages + 2;        // tile accumulators in flight (see the epilogue)
  int off = stages * L.stage_bytes;
  L.x_off = off;
  off += T * (K * 2 + 16);
  off = (off + 15) & ~15;
  L.zero_off = off;
  off += 16;
  L.acc_off = off;
  off += L.nbuf * 8 * kTileRows * T * 4;  // [nbuf][warp (<= 8)][16][T] partial tiles
  L.cnt_off = off;
  off += L.nbuf * 4;
  off = (off + 7) & ~7;
  L.bar_off = off;
  off += 2 * stages * 8;
  L.misc_off = off;
  off += 64;
  L.down_off = off;
  off += down_floats * 4;
  L.total = off + 128;
  return L;
}

// down[t][r] = x_staged[t] . A[adapter(t)][r] (fp32) for every token of the
// launch, into shared memory; `scratch` holds [warps][T][rank] partials (the
// tile-accumulator region, unused until the main loop).  rank <= 64.
__device__ __forceinline__ void down_from_staged(const GemvArgs& a, const uint8_t* xs, int xrow, float* down,
                                                 float* scratch, int tid, int nthreads, int bar) {
  const int K = a.K, R = a.rank;
  const int lane = tid & 31, wid = tid >> 5, nw = nthreads >> 5;
  for (int t = 0; t < a.T; ++t) {
    const int ad = a.tok_adapter != nullptr ? a.tok_adapter[t] : 0;
    if (ad < 0 || ad >= a.pro_a_adapters) continue;  // no LoRA for this token: its down is not read
    const bf16* A = a.pro_a + (int64_t)ad * R * K;
    const uint8_t* xr = xs + t * xrow;
    for (int r0 = 0; r0 < R; r0 += 16) {
      float acc[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = 0.f;
      for (int k = tid * 8; k < K; k += nthreads * 8) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xr + k * 2);
        const uint32_t* xu = reinterpret_cast<const uint32_t*>(&xv);
        float xf[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(xu[q]);
          xf[2 * q] = f.x;
          xf[2 * q + 1] = f.y;
        }
        uint4 av[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          av[i] = r0 + i < R ? __ldg(reinterpret_cast<const uint4*>(A + (int64_t)(r0 + i) * K + k))
                             : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t* au = reinterpret_cast<const uint32_t*>(&av[i]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = unpack_bf16x2(au[q]);
            acc[i] = fmaf(xf[2 * q], f.x, acc[i]);
            acc[i] = fmaf(xf[2 * q + 1], f.y, acc[i]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float v = warp_sum(acc[i]);
        if (lane == 0 && r0 + i < R) scratch[(wid * a.T + t) * R + r0 + i] = v;
      }
    }
  }
  named_barrier(bar, nthreads);
  for (int i = tid; i < a.T * R; i += nthreads) {
    float v = 0.f;
    for (int w = 0; w < nw; ++w) v += scratch[w * a.T * R + i];  // fixed order
    down[i] = v;
  }
  named_barrier(bar, nthreads);
}

// Stage the activations of all tokens as bf16 rows (stride xrow bytes) in
// shared memory, applying the input prologue.  Loads are issued four chunks
// at a time per thread so each pass costs one or two memory round trips.
// kCg: the activations were written by other CTAs of the same launch (read
// them from L2).
// `part` holds one float per warp; `bar` is a named barrier over `nthreads`.
template <bool kCg = false>
__device__ __forceinline__ void stage_activations(const GemvArgs& a, uint8_t* xs, int xrow, int tid, int nthreads,
                                                  float* part, int bar) {
  const int K = a.K;
  const int lane = tid & 31, wid = tid >> 5;
  const int step = nthreads * 8;
  for (int t = 0; t < a.T; ++t) {
    const bf16* xr = a.x + (int64_t)t * a.x_stride;
    uint8_t* dst = xs + t * xrow;
    if (a.prologue == PL_PROLOGUE_RMSNORM && K <= 4 * step) {
      // one pass: x and the norm weights stay in registers across the
      // reduction (same sum order as the two-pass form below)
      uint4 v[4], wv[4];
      const int k0 = tid * 8;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = k0 + i * step;
        v[i] = k < K ? ld_act16<kCg>(xr + k) : make_uint4(0, 0, 0, 0);
        wv[i] = k < K ? *reinterpret_cast<const uint4*>(a.norm_w + k) : make_uint4(0, 0, 0, 0);
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(u[q]);
          ss += f.x * f.x + f.y * f.y;
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) part[wid] = ss;
      named_barrier(bar, nthreads);
      float tot = 0.f;
      for (int w = 0; w < nthreads / 32; ++w) tot += part[w];
      const float rstd = rsqrtf(tot / (float)K + a.eps);
      named_barrier(bar, nthreads);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int k = k0 + i * step;
        if (k >= K) break;
        const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
        const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv[i]);
        uint4 o;
        uint32_t* uo = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(u[q]);
          const float2 g = unpack_bf16x2(uw[q]);
          uo[q] = pack_bf16x2(f.x * rstd * g.x, f.y * rstd * g.y);
        }
        *reinterpret_cast<uint4*>(dst + k * 2) = o;
      }
    } else if (a.prologue == PL_PROLOGUE_RMSNORM) {
      float ss = 0.f;
      for (int k0 = tid * 8; k0 < K; k0 += 4 * step) {
        uint4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = k0 + i * step;
          v[i] = k < K ? ld_act16<kCg>(xr + k) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = unpack_bf16x2(u[q]);
            ss += f.x * f.x + f.y * f.y;
          }
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) part[wid] = ss;
      named_barrier(bar, nthreads);
      float tot = 0.f;
      for (int w = 0; w < nthreads / 32; ++w) tot += part[w];
      const float rstd = rsqrtf(tot / (float)K + a.eps);
      named_barrier(bar, nthreads);
      for (int k0 = tid * 8; k0 < K; k0 += 4 * step) {
        uint4 v[4], wv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = k0 + i * step;
          v[i] = k < K ? ld_act16<kCg>(xr + k) : make_uint4(0, 0, 0, 0);
          wv[i] = k < K ? *reinterpret_cast<const uint4*>(a.norm_w + k) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = k0 + i * step;
          if (k >= K) break;
          const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
          const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv[i]);
          uint4 o;
          uint32_t* uo = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = unpack_bf16x2(u[q]);
            const float2 g = unpack_bf16x2(uw[q]);
            uo[q] = pack_bf16x2(f.x * rstd * g.x, f.y * rstd * g.y);
          }
          *reinterpret_cast<uint4*>(dst + k * 2) = o;
        }
      }
    } else if (a.prologue == PL_PROLOGUE_SILU_MUL) {
      for (int k0 = tid * 8; k0 < K; k0 += 4 * step) {
        uint4 gv[4], uv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = k0 + i * step;
          gv[i] = k < K ? ld_act16<kCg>(xr + k) : make_uint4(0, 0, 0, 0);
          uv[i] = k < K ? ld_act16<kCg>(xr + K + k) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = k0 + i * step;
          if (k >= K) break;
          const uint32_t* ug = reinterpret_cast<const uint32_t*>(&gv[i]);
          const uint32_t* uu = reinterpret_cast<const uint32_t*>(&uv[i]);
          uint4 o;
          uint32_t* uo = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 g = unpack_bf16x2(ug[q]);
            const float2 up = unpack_bf16x2(uu[q]);
            uo[q] = pack_bf16x2(silu_mul(g.x, up.x), silu_mul(g.y, up.y));
          }
          *reinterpret_cast<uint4*>(dst + k * 2) = o;
        }
      }
    } else {
      for (int k0 = tid * 8; k0 < K; k0 += 4 * step) {
        uint4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = k0 + i * step;
          v[i] = k < K ? ld_act16<kCg>(xr + k) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int k = k0 + i * step;
          if (k < K) *reinterpret_cast<uint4*>(dst + k * 2) = v[i];
        }
      }
    }
  }
  named_barrier(bar, nthreads);
}

// Shared-memory pieces of one GEMV CTA (linear_lora_kernel, linear_chain_kernel).
struct GemvRing {
  uint8_t* smem;
  GemvSmem L;
  uint64_t* full_bar;
  uint64_t* empty_bar;
  volatile int32_t* abort_flag;
  float* tacc;    // [nbuf][NCW][16][T] partial tiles
  int32_t* tcnt;  // [nbuf] warps done with a tile
  uint8_t* xs;    // staged activations
  int S, KC;
};

__device__ __forceinline__ GemvRing gemv_ring(uint8_t* smem_raw, const GemvSmem& L, int S, int KC) {
  GemvRing R;
  R.smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  R.L = L;
  R.full_bar = reinterpret_cast<uint64_t*>(R.smem + L.bar_off);
  R.empty_bar = R.full_bar + S;
  R.abort_flag = reinterpret_cast<volatile int32_t*>(R.smem + L.misc_off);
  R.tacc = reinterpret_cast<float*>(R.smem + L.acc_off);
  R.tcnt = reinterpret_cast<int32_t*>(R.smem + L.cnt_off);
  R.xs = R.smem + L.x_off;
  R.S = S;
  R.KC = KC;
  return R;
}

// Barriers, tile counters and the zero slot; ends with a CTA barrier.
template <int NCW>
__device__ __forceinline__ void gemv_ring_init(const GemvRing& R) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < R.S; ++s) {
      mbar_init(&R.full_bar[s], 1);
      mbar_init(&R.empty_bar[s], NCW);
    }
    *R.abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < R.L.nbuf; i += blockDim.x) R.tcnt[i] = 0;
  if (threadIdx.x < 4) reinterpret_cast<uint32_t*>(R.smem + R.L.zero_off)[threadIdx.x] = 0u;
  __syncthreads();
}

// Producer warp: stream the 16-row x kc-column tiles of weight rows [r0, r1)
// into the ring as ring units u_base, u_base + 1, ...  Lane r issues the
// bulk copy of row r's kc columns, because a TMA instruction costs ~0.3 us
// of issue time however many lanes take part.  Returns the units issued
// (fewer after an abort).
__device__ __forceinline__ int gemv_produce(const GemvArgs& a, const GemvRing& R, int64_t r0, int64_t r1, int u_base,
                                            uint64_t pol, int lane) {
  const int S = R.S, KC = R.KC, K = a.K;
  const int n_tiles = (int)((r1 - r0 + kTileRows - 1) / kTileRows);
  const int n_kc = (K + KC - 1) / KC;
  const int n_units = n_tiles * n_kc;
  const int RB = R.L.row_bytes;
  int issued = 0;
  for (int lu = 0; lu < n_units; ++lu) {
    const int u = u_base + lu;
    const int s = u % S;
    if (u >= S) {
      if (!mbar_wait(&R.empty_bar[s], ((u / S) - 1) & 1)) {
        if (lane == 0) {
          set_status(a.status, PL_ERR_TIMEOUT);
          *R.abort_flag = 1;
        }
      }
    }
    __syncwarp();
    if (*R.abort_flag) break;
    const int tile = lu / n_kc, kc = lu % n_kc;
    const int64_t row0 = r0 + (int64_t)tile * kTileRows;
    const int rows = (int)((r1 - row0) < kTileRows ? (r1 - row0) : kTileRows);
    const int k0 = kc * KC;
    const int kw = min(KC, K - k0);
    if (lane == 0) mbar_arrive_expect_tx(&R.full_bar[s], (uint32_t)(rows * kw * 2));
    __syncwarp();
    if (lane < rows) {
      const int64_t row = row0 + lane;
      const bf16* src = row < a.n_out ? a.w + row * K : a.shrink_a + (row - a.n_out) * K;
      bulk_g2s(R.smem + s * R.L.stage_bytes + lane * RB, src + k0, (uint32_t)(kw * 2), &R.full_bar[s], pol);
    }
    if (lane == 0 && u == 0) PL_TRACE_POINT(1);
    if (lane == 0 && u == S) PL_TRACE_POINT(2);
    ++issued;
  }
  return issued;
}

// After an abort: wait (bounded) for the copies still in flight, the last
// min(issued, S) units, so that no TMA write lands after the CTA exits.
__device__ __forceinline__ void gemv_drain(const GemvRing& R, int issued) {
  for (int u = issued - R.S < 0 ? 0 : issued - R.S; u < issued; ++u)
    (void)mbar_wait(&R.full_bar[u % R.S], (u / R.S) & 1);
}

// After this CTA's own copies: pull into L2 the first pf_units ring units
// (16 rows x pf_kc columns each) that CTA blockIdx.x of the NEXT projection
// will load, so that launch's first stages come from L2 instead of DRAM.
__device__ __forceinline__ void gemv_prefetch_next(const GemvArgs& a, int lane) {
  if (a.pf_units <= 0 || (int)blockIdx.x >= a.pf_grid) return;
  const int64_t r0 = a.pf_rows_total * blockIdx.x / a.pf_grid;
  const int64_t r1 = a.pf_rows_total * (blockIdx.x + 1) / a.pf_grid;
  const int n_kc = (a.pf_k + a.pf_kc - 1) / a.pf_kc;
  for (int u = 0; u < a.pf_units; ++u) {
    const int64_t row0 = r0 + (int64_t)(u / n_kc) * kTileRows;
    if (row0 >= r1) break;
    const int k0 = (u % n_kc) * a.pf_kc;
    const int kw = min(a.pf_kc, a.pf_k - k0);
    const int64_t row = row0 + lane;
    if (lane < kTileRows && row < r1) {
      const bf16* src = row < a.pf_n_out ? a.pf_w + row * a.pf_k : a.pf_shrink + (row - a.pf_n_out) * a.pf_k;
      bulk_prefetch_l2(src + k0, (uint32_t)kw * 2);
    }
  }
}

// Consumer warps: multiply the ring units u_base, ... (weight rows [r0, r1)
// of one projection) against the staged activations with mma.sync
// m16n8k16 (weight rows = M, tokens = N); the warps split the k-steps of
// each stage, and at the end of a tile each warp stores its partial tile
// in its own slot and the last warp to arrive sums the slots in warp order
// (deterministic) and runs the epilogue, so no CTA-wide barrier ever stalls
// the stream.  Returns false after an abort.
template <int NCW>
__device__ __forceinline__ bool gemv_consume(const GemvArgs& a, const GemvRing& R, int64_t r0, int64_t r1, int u_base,
                                             const float* down, int64_t dstride, int cw, int ctid, int lane,
                                             bool trace = true) {
  const int S = R.S, KC = R.KC, K = a.K;
  const int n_tiles = (int)((r1 - r0 + kTileRows - 1) / kTileRows);
  const int n_kc = (K + KC - 1) / KC;
  const int n_units = n_tiles * n_kc;
  const int RB = R.L.row_bytes;
  const int XROW = K * 2 + 16;
  const int g = lane >> 2, tq = lane & 3;
  const uint32_t zero_addr = smem_u32(R.smem + R.L.zero_off);
  // Per-lane ldmatrix row addresses.
  const int a_row = (lane & 7) + 8 * ((lane >> 3) & 1);
  const int a_col = 8 * (lane >> 4);
  const int b_tok = lane & 7;
  const int b_col = 8 * ((lane >> 3) & 1);
  const bool b_valid = b_tok < a.T;
  const uint32_t xs_base = smem_u32(R.xs + b_tok * XROW + b_col * 2);

  for (int tile = 0; tile < n_tiles; ++tile) {
    // two independent accumulators so consecutive mma's do not serialise
    float acc0[4] = {0.f, 0.f, 0.f, 0.f};
    float acc1[4] = {0.f, 0.f, 0.f, 0.f};
    for (int kc = 0; kc < n_kc; ++kc) {
      const int lu = tile * n_kc + kc;
      const int u = u_base + lu;
      const int s = u % S;
      if (!mbar_wait(&R.full_bar[s], (u / S) & 1)) {
        if (lane == 0) set_status(a.status, PL_ERR_TIMEOUT);
        *R.abort_flag = 1;
      }
      if (*R.abort_flag) return false;
      if (trace && ctid == 0 && u == 0) PL_TRACE_POINT(6);
      if (trace && ctid == 0 && lu == n_units - 1) PL_TRACE_POINT(7);
      const int k0 = kc * KC;
      const int ksteps = min(KC, K - k0) / 16;
      const uint32_t stage = smem_u32(R.smem + s * R.L.stage_bytes) + a_row * RB + a_col * 2;
      const uint32_t xcol = xs_base + k0 * 2;
      for (int ks = cw; ks < ksteps; ks += 2 * NCW) {
        const bool two = ks + NCW < ksteps;
        uint32_t a0[4], b0[2], a1[4], b1[2];
        ldsm_x4(stage + ks * 32, a0[0], a0[1], a0[2], a0[3]);
        ldsm_x2(b_valid ? xcol + ks * 32 : zero_addr, b0[0], b0[1]);
        if (two) {
          ldsm_x4(stage + (ks + NCW) * 32, a1[0], a1[1], a1[2], a1[3]);
          ldsm_x2(b_valid ? xcol + (ks + NCW) * 32 : zero_addr, b1[0], b1[1]);
        }
        mma_bf16_16816(acc0, a0, b0);
        if (two) mma_bf16_16816(acc1, a1, b1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&R.empty_bar[s]);
    }
    const int T = a.T;
    const int buf = tile % R.L.nbuf;
    float* slots = R.tacc + buf * (NCW * kTileRows * T);
    float* mine = slots + cw * (kTileRows * T);
    if (2 * tq < T) {
      mine[g * T + 2 * tq] = acc0[0] + acc1[0];
      mine[(g + 8) * T + 2 * tq] = acc0[2] + acc1[2];
    }
    if (2 * tq + 1 < T) {
      mine[g * T + 2 * tq + 1] = acc0[1] + acc1[1];
      mine[(g + 8) * T + 2 * tq + 1] = acc0[3] + acc1[3];
    }
    __threadfence_block();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = (atomicAdd(&R.tcnt[buf], 1) == NCW - 1);
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence_block();
      for (int e = lane; e < kTileRows * T; e += 32) {
        const int row = e / T, tok = e % T;
        const int64_t o = r0 + (int64_t)tile * kTileRows + row;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < NCW; ++w) v += *reinterpret_cast<volatile float*>(&slots[w * kTileRows * T + e]);
        if (o < r1) gemv_epilogue(a, o, tok, v, down, dstride);
      }
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        R.tcnt[buf] = 0;
      }
    }
  }
  return true;
}

// Stage the activations (and the in-kernel LoRA down) of one projection;
// returns the down rows the epilogue reads.
template <bool kCg>
__device__ __forceinline__ const float* gemv_stage(const GemvArgs& a, const GemvRing& R, int ctid, int nc,
                                                   int64_t& dstride) {
  const int XROW = a.K * 2 + 16;
  stage_activations<kCg>(a, R.xs, XROW, ctid, nc, reinterpret_cast<float*>(R.smem + R.L.misc_off + 16), 1);
  dstride = a.down_stride;
  if (a.pro_a == nullptr) return a.lora_down;
  float* dsm = reinterpret_cast<float*>(R.smem + R.L.down_off);
  down_from_staged(a, R.xs, XROW, dsm, R.tacc, ctid, nc, 1);
  dstride = a.rank;
  return dsm;
}

// One CTA per SM streams the weight rows [r0, r1) of its balanced share as
// 16-row x kc-column tiles through an S-deep shared-memory ring (one
// producer warp, NCW consumer warps).
template <int NCW>
__global__ void __launch_bounds__(32 * (1 + NCW), 1) linear_lora_kernel(const GemvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const GemvSmem L = gemv_smem_layout(a.T, a.K, a.stages, a.kc, a.pro_a != nullptr ? a.T * a.rank : 0);
  const GemvRing R = gemv_ring(smem_raw, L, a.stages, a.kc);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t rows_total = (int64_t)a.n_out + a.n_shrink;
  const int64_t r0 = rows_total * blockIdx.x / gridDim.x;
  const int64_t r1 = rows_total * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) PL_TRACE_POINT(0);
  gemv_ring_init<NCW>(R);
  pdl_launch_dependents();

  if (warp == 0) {
    // --------------------------------------------------------- producer warp
    if (!a.early_weights) pdl_wait();
    const int issued = gemv_produce(a, R, r0, r1, 0, l2_evict_first_policy(), lane);
    if (!*R.abort_flag) gemv_prefetch_next(a, lane);
    if (lane == 0) PL_TRACE_POINT(3);
    if (lane == 0 && *R.abort_flag) gemv_drain(R, issued);
    return;
  }

  // ------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int ctid = threadIdx.x - 32;
  pdl_wait();
  if (ctid == 0) PL_TRACE_POINT(4);
  int64_t dstride;
  const float* down = gemv_stage<false>(a, R, ctid, 32 * NCW, dstride);
  if (ctid == 0) PL_TRACE_POINT(5);
  gemv_consume<NCW>(a, R, r0, r1, 0, down, dstride, cw, ctid, lane);
  if (lane == 0) PL_TRACE_MAX(8);
}

// ------------------------------------------------------- projection chain
// Up to kMaxChainPhases projections in one persistent launch (one CTA per
// SM, all resident), e.g. o -> gate_up -> down -> the next layer's q/k/v.
// The producer warp streams the weights of every phase back to back through
// one ring: the weights depend on nothing upstream, so the ring keeps
// filling while the consumers of phase p wait for the outputs of phase p-1.
// Between phases the consumer warps of all CTAs meet at a grid barrier (a
// global arrival counter; bounded wait); the activations and residuals
// written inside the launch are then read from L2.  The counter resets
// itself: each CTA adds one more arrival after passing the last barrier and
// the CTA that brings the count to num_phases x grid puts it back to zero.
// Trace points (-DPL_TRACE builds): 0 start, 1 / 2 producer issued unit 0 /
// unit S, 3 producer done, 4 consumers past the upstream wait, 5 phase-0
// activations staged, 6 + p phase p's tiles done (p < 4), 10 + p grid
// barrier before phase p passed (p = 1..3), 14 phase-1 activations staged,
// 15 last consumer warp done.
constexpr int kMaxChainPhases = 6;

struct GemvChainArgs {
  GemvArgs ph[kMaxChainPhases];
  int32_t num_phases;
  int32_t stages, kc, k_max, down_max;
  int32_t* barrier;
  int32_t* status;
};

__device__ __forceinline__ void red_release_gpu_add(int32_t* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier of the consumer warps: all CTAs have finished the phases
// before `target / gridDim.x`.  Every consumer thread calls it (a warp that
// gave up in the previous phase too), and all of them get the same answer:
// thread 0 decides and broadcasts it through shared memory, so either every
// consumer warp goes on to the next phase's named barriers or none does.
// False on timeout or after an abort anywhere in the CTA (status set).
__device__ __forceinline__ bool chain_grid_barrier(const GemvChainArgs& c, const GemvRing& R, int target, int ctid,
                                                   int nc) {
  volatile int32_t* go = reinterpret_cast<volatile int32_t*>(R.smem + R.L.misc_off + 4);
  named_barrier(1, nc);  // every epilogue store of this CTA's phase is issued
  if (ctid == 0) {
    bool ok = *R.abort_flag == 0;
    if (ok) {
      // release: this CTA's stores (ordered before by the named barrier) are
      // visible to whoever acquires the count; acquire: the other CTAs' are
      // visible here, and through the named barrier below to every warp
      red_release_gpu_add(c.barrier, 1);
      const long long c0 = clock64();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire_gpu(c.barrier) >= target) break;
        if ((i & 255u) == 0 && clock64() - c0 > kWaitTimeoutCycles) {
          set_status(c.status, PL_ERR_TIMEOUT);
          *R.abort_flag = 1;
          ok = false;
          break;
        }
      }
    }
    *go = ok ? 1 : 0;
  }
  named_barrier(1, nc);
  return *go != 0;
}

template <int NCW>
__global__ void __launch_bounds__(32 * (1 + NCW), 1) linear_chain_kernel(const __grid_constant__ GemvChainArgs c) {
  extern __shared__ uint8_t smem_raw[];
  const GemvSmem L = gemv_smem_layout(c.ph[0].T, c.k_max, c.stages, c.kc, c.down_max);
  const GemvRing R = gemv_ring(smem_raw, L, c.stages, c.kc);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int G = gridDim.x;

  if (threadIdx.x == 0) PL_TRACE_POINT(0);
  gemv_ring_init<NCW>(R);
  pdl_launch_dependents();

  if (warp == 0) {
    // Producer: every phase's weights, back to back (static: no upstream wait).
    const uint64_t pol = l2_evict_first_policy();
    int u_base = 0;
    for (int p = 0; p < c.num_phases; ++p) {
      const GemvArgs& a = c.ph[p];
      const int64_t rows_total = (int64_t)a.n_out + a.n_shrink;
      const int64_t r0 = rows_total * blockIdx.x / G, r1 = rows_total * (blockIdx.x + 1) / G;
      const int n_units = (int)((r1 - r0 + kTileRows - 1) / kTileRows) * ((a.K + R.KC - 1) / R.KC);
      const int issued = gemv_produce(a, R, r0, r1, u_base, pol, lane);
      if (issued < n_units) {
        if (lane == 0) gemv_drain(R, u_base + issued);
        return;
      }
      u_base += n_units;
    }
    if (lane == 0) PL_TRACE_POINT(3);
    // no copy may land after the CTA exits (the consumers can stop early)
    if (lane == 0) gemv_drain(R, u_base);
    return;
  }

  const int cw = warp - 1;
  const int ctid = threadIdx.x - 32;
  constexpr int NC = 32 * NCW;
  pdl_wait();  // phase 0's activations come from the upstream kernel
  if (ctid == 0) PL_TRACE_POINT(4);
  int u_base = 0;
  for (int p = 0; p < c.num_phases; ++p) {
    const GemvArgs& a = c.ph[p];
    if (p > 0 && !chain_grid_barrier(c, R, p * G, ctid, NC)) break;
    if (ctid == 0 && p > 0 && p < 4) PL_TRACE_POINT(10 + p);
    if (c.num_phases > 1 && p == c.num_phases - 1 && ctid == 0) {
      // past the last barrier: the extra arrival that lets the counter reset
      if (atomicAdd(c.barrier, 1) == c.num_phases * G - 1) atomicExch(c.barrier, 0);
    }
    const int64_t rows_total = (int64_t)a.n_out + a.n_shrink;
    const int64_t r0 = rows_total * blockIdx.x / G, r1 = rows_total * (blockIdx.x + 1) / G;
    int64_t dstride;
    const float* down = gemv_stage<true>(a, R, ctid, NC, dstride);
    if (ctid == 0 && p < 2) PL_TRACE_POINT(p == 0 ? 5 : 14);
    // a warp that gives up (bounded wait) still meets the others at the next
    // grid barrier, which then stops every warp of the CTA together
    (void)gemv_consume<NCW>(a, R, r0, r1, u_base, down, dstride, cw, ctid, lane, false);
    if (ctid == 0 && p < 4) PL_TRACE_POINT(6 + p);
    u_base += (int)((r1 - r0 + kTileRows - 1) / kTileRows) * ((a.K + R.KC - 1) / R.KC);
  }
  if (lane == 0) PL_TRACE_MAX(15);
}

// ------------------------------------------------- register-direct variant
// Each CTA owns 16-row tiles (strided over the grid); its warps split K into
// 32-column blocks.  A thread loads 16 bytes of weight row g and of row g+8
// per block straight into registers (no shared-memory staging, no TMA issue
// cost) and feeds them to mma.sync as A fragments with the 32 columns of the
// block permuted: the k-step pairs {2t, 2t+1, 2t+8, 2t+9} map to columns
// {8t .. 8t+3} and the second k-step to {8t+4 .. 8t+7}.  The activations use
// the same mapping (one 16-byte shared load per block); a dot product does
// not depend on the order of its k terms, so the permutation is free.  Loads run
// one batch of kLdgUnroll blocks ahead of the math; the first batch of the
// first tile is requested before the upstream grid has finished (static
// weights).  Partial tiles of the warps are combined in shared memory.
constexpr int kLdgUnroll = 4;

struct LdgSmem {
  int xrow, red_off, part_off, zero_off, total;
};
__host__ __device__ inline LdgSmem ldg_smem_layout(int T, int K, int nw) {
  LdgSmem L;
  L.xrow = K * 2 + 16;
  int off = T * L.xrow;
  off = (off + 15) & ~15;
  L.red_off = off;
  off += 2 * nw * kTileRows * kMaxTok * 4;
  L.part_off = off;
  off += 64;
  L.zero_off = off;
  off += 16;
  L.total = off + 128;
  return L;
}

template <int NW>
__global__ void __launch_bounds__(32 * NW) linear_ldg_kernel(const GemvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int K = a.K, T = a.T;
  const LdgSmem L = ldg_smem_layout(T, K, NW);
  uint8_t* xs = smem;
  float* red = reinterpret_cast<float*>(smem + L.red_off);  // [2][NW][16][8]
  float* part = reinterpret_cast<float*>(smem + L.part_off);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = lane >> 2, tq = lane & 3;
  const int64_t rows_total = (int64_t)a.n_out + a.n_shrink;
  const int n_tiles = (int)((rows_total + kTileRows - 1) / kTileRows);
  const int nblk = K / 32;
  const int b0 = warp * nblk / NW, b1 = (warp + 1) * nblk / NW;
  if (threadIdx.x < 4) reinterpret_cast<uint32_t*>(smem + L.zero_off)[threadIdx.x] = 0u;
  if (threadIdx.x == 0) PL_TRACE_POINT(0);
  pdl_launch_dependents();

  auto row_ptr = [&](int64_t row) -> const uint4* {
    const bf16* p = row < a.n_out ? a.w + row * K : a.shrink_a + (row - a.n_out) * K;
    return reinterpret_cast<const uint4*>(p) + tq;  // this lane's 16 bytes of each 32-column block
  };
  // Weight registers of one batch of blocks: rows g and g + 8.
  uint4 wa[kLdgUnroll], wb[kLdgUnroll];
  auto load_batch = [&](int tile, int bb) {
    const int64_t ra = (int64_t)tile * kTileRows + g, rb = ra + 8;
    const bool va = ra < rows_total, vb = rb < rows_total;
    const uint4* pa = row_ptr(va ? ra : 0);
    const uint4* pb = row_ptr(vb ? rb : 0);
#pragma unroll
    for (int u = 0; u < kLdgUnroll; ++u) {
      const int blk = bb + u;
      const bool in = blk < b1;
      wa[u] = (in && va) ? __ldcs(pa + blk * 4) : make_uint4(0, 0, 0, 0);
      wb[u] = (in && vb) ? __ldcs(pb + blk * 4) : make_uint4(0, 0, 0, 0);
    }
  };

  int tile = blockIdx.x;
  if (a.early_weights && warp == 0) {
    // Pull the weights of this CTA's first tiles into L2 while the upstream
    // grid is still running (16 KB per lane request; a tile is contiguous).
    for (int j = 0; j < a.prefetch_tiles; ++j) {
      const int t = blockIdx.x + j * (int)gridDim.x;
      if (t >= n_tiles) break;
      int64_t r0 = (int64_t)t * kTileRows, r1 = r0 + kTileRows;
      if (r1 > rows_total) r1 = rows_total;
      for (int part_i = 0; part_i < 2; ++part_i) {
        const int64_t lo = part_i == 0 ? r0 : (r0 > a.n_out ? r0 : (int64_t)a.n_out);
        const int64_t hi = part_i == 0 ? (r1 < a.n_out ? r1 : (int64_t)a.n_out) : r1;
        if (hi <= lo) continue;
        const char* base = part_i == 0 ? reinterpret_cast<const char*>(a.w + lo * K)
                                       : reinterpret_cast<const char*>(a.shrink_a + (lo - a.n_out) * K);
        const int64_t bytes = (hi - lo) * K * 2;
        for (int64_t off = (int64_t)lane * 16384; off < bytes; off += 32 * 16384) {
          const int64_t left = bytes - off;
          prefetch_l2_bulk(base + off, (uint32_t)(left < 16384 ? left : 16384));
        }
      }
    }
  }
  if (a.early_weights && tile < n_tiles && b0 < b1) load_batch(tile, b0);
  pdl_wait();
  if (!a.early_weights && tile < n_tiles && b0 < b1) load_batch(tile, b0);
  stage_activations(a, xs, L.xrow, threadIdx.x, 32 * NW, part, 1);
  if (threadIdx.x == 0) PL_TRACE_POINT(5);

  const uint32_t zero_addr = smem_u32(smem + L.zero_off);
  const uint32_t xbase = g < T ? smem_u32(xs + g * L.xrow) + tq * 16 : 0u;
  for (int it = 0; tile < n_tiles; tile += gridDim.x, ++it) {
    float acc0[4] = {0.f, 0.f, 0.f, 0.f};
    float acc1[4] = {0.f, 0.f, 0.f, 0.f};
    for (int bb = b0; bb < b1; bb += kLdgUnroll) {
      uint4 ca[kLdgUnroll], cb[kLdgUnroll];
#pragma unroll
      for (int u = 0; u < kLdgUnroll; ++u) {
        ca[u] = wa[u];
        cb[u] = wb[u];
      }
      // request the next batch (this tile's next blocks, or the next tile's first)
      if (bb + kLdgUnroll < b1)
        load_batch(tile, bb + kLdgUnroll);
      else if (tile + (int)gridDim.x < n_tiles)
        load_batch(tile + gridDim.x, b0);
#pragma unroll
      for (int u = 0; u < kLdgUnroll; ++u) {
        const int blk = bb + u;
        if (blk < b1) {
          uint32_t xv[4];
          const uint32_t xaddr = g < T ? xbase + blk * 64 : zero_addr;
          asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(xv[0]), "=r"(xv[1]), "=r"(xv[2]), "=r"(xv[3])
                       : "r"(xaddr));
          const uint32_t a0[4] = {ca[u].x, cb[u].x, ca[u].y, cb[u].y};
          const uint32_t a1[4] = {ca[u].z, cb[u].z, ca[u].w, cb[u].w};
          mma_bf16_16816(acc0, a0, &xv[0]);
          mma_bf16_16816(acc1, a1, &xv[2]);
        }
      }
    }
    // combine the warps' partial tiles, then the epilogue of the tile
    float* rb = red + (it & 1) * (NW * kTileRows * kMaxTok);
    float* mine = rb + warp * (kTileRows * kMaxTok);
    mine[g * kMaxTok + 2 * tq] = acc0[0] + acc1[0];
    mine[g * kMaxTok + 2 * tq + 1] = acc0[1] + acc1[1];
    mine[(g + 8) * kMaxTok + 2 * tq] = acc0[2] + acc1[2];
    mine[(g + 8) * kMaxTok + 2 * tq + 1] = acc0[3] + acc1[3];
    __syncthreads();
    for (int e = threadIdx.x; e < kTileRows * T; e += 32 * NW) {
      const int row = e / T, tok = e % T;
      const int64_t o = (int64_t)tile * kTileRows + row;
      if (o < rows_total) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) v += rb[(w * kTileRows + row) * kMaxTok + tok];
        gemv_epilogue(a, o, tok, v);
      }
    }
  }
  if (threadIdx.x == 0) PL_TRACE_MAX(8);
}

// ----------------------------------------------------------------- shrink
// One CTA per (rank row j, segment); down[t, j] = x[t] . A[adapter][j].
__global__ void __launch_bounds__(256) lora_shrink_kernel(const bf16* __restrict__ x, int64_t x_stride,
                                                         const bf16* __restrict__ A, int num_adapters, int rank,
                                                         int K, const int32_t* __restrict__ seg_indptr,
                                                         const int32_t* __restrict__ seg_adapter,
                                                         float* __restrict__ down, int64_t down_stride) {
  pdl_launch_dependents();
  pdl_wait();
  const int j = blockIdx.x, sg = blockIdx.y;
  const int t0 = seg_indptr[sg], t1 = seg_indptr[sg + 1];
  const int ad = seg_adapter[sg];
  __shared__ float part[8][kMaxTok];
  if (ad < 0 || ad >= num_adapters) {
    for (int t = t0 + threadIdx.x; t < t1; t += blockDim.x) down[t * down_stride + j] = 0.f;
    return;
  }
  const bf16* arow = A + ((int64_t)ad * rank + j) * K;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  for (int tb = t0; tb < t1; tb += kMaxTok) {
    const int nt = min(kMaxTok, t1 - tb);
    float acc[kMaxTok];
#pragma unroll
    for (int i = 0; i < kMaxTok; ++i) acc[i] = 0.f;
    for (int k = threadIdx.x * 8; k < K; k += blockDim.x * 8) {
      uint4 av = *reinterpret_cast<const uint4*>(arow + k);
      const uint32_t* ua = reinterpret_cast<const uint32_t*>(&av);
      float af[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float2 f = unpack_bf16x2(ua[i]);
        af[2 * i] = f.x;
        af[2 * i + 1] = f.y;
      }
#pragma unroll
      for (int i = 0; i < kMaxTok; ++i) {
        if (i < nt) {
          uint4 xv = *reinterpret_cast<const uint4*>(x + (int64_t)(tb + i) * x_stride + k);
          const uint32_t* ux = reinterpret_cast<const uint32_t*>(&xv);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float2 f = unpack_bf16x2(ux[q]);
            acc[i] += af[2 * q] * f.x + af[2 * q + 1] * f.y;
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kMaxTok; ++i) {
      float v = warp_sum(acc[i]);
      if (lane == 0) part[warp][i] = v;
    }
    __syncthreads();
    if (threadIdx.x < nt) {
      float v = 0.f;
      for (int w = 0; w < (int)(blockDim.x / 32); ++w) v += part[w][threadIdx.x];
      down[(int64_t)(tb + threadIdx.x) * down_stride + j] = v;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------- row shrink
// down[t][j] = row_t . A[adapter(t)][j] for rank rows j of one block: CTA
// (t, jb) takes token t and rank rows [4 jb, 4 jb + 4).  The token's row is
// loaded once into registers (thread `tid` holds the 8-element chunks
// k = tid * 8 + i * 2048, i < 4, so K <= 8192), optionally RMS-normalised
// first with the partition and sum order of rmsnorm_kernel (so the
// normalised row is bit-identical to pl_rmsnorm's; every CTA of the token
// recomputes the norm and the jb == 0 CTA writes the row out), then the
// CTA's four A rows (requested together with the row) are reduced by warp
// shuffles and the 8 warps' sums in warp order.  The A rows are spread over
// T x R/4 CTAs, so the launch has enough CTAs to read them in parallel.
constexpr int kShrinkThreads = 256;
constexpr int kShrinkChunks = 4;
constexpr int kShrinkRowsPerCta = 4;

__global__ void __launch_bounds__(kShrinkThreads, 2) lora_shrink_rows_kernel(
    const bf16* __restrict__ x, int64_t x_stride, int K, const bf16* __restrict__ norm_w, float eps,
    bf16* __restrict__ xn, int64_t xn_stride, const bf16* __restrict__ A, int num_adapters, int R,
    const int32_t* __restrict__ tok_adapter, float* __restrict__ down, int64_t down_stride) {
  __shared__ float part[kShrinkThreads / 32][kShrinkRowsPerCta];
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x, j0 = blockIdx.y * kShrinkRowsPerCta;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  constexpr int kStep = kShrinkThreads * 8;
  const int ad = tok_adapter != nullptr ? tok_adapter[t] : 0;
  const bool lora = ad >= 0 && ad < num_adapters;
  const bf16* xr = x + (int64_t)t * x_stride;
  const bf16* Aad = A + (int64_t)(lora ? ad : 0) * R * K;
  uint4 v[kShrinkChunks], av[kShrinkRowsPerCta][kShrinkChunks];
#pragma unroll
  for (int i = 0; i < kShrinkChunks; ++i) {
    const int k = tid * 8 + i * kStep;
    v[i] = k < K ? *reinterpret_cast<const uint4*>(xr + k) : make_uint4(0, 0, 0, 0);
  }
  // the A rows do not depend on the row: requested with it
#pragma unroll
  for (int jj = 0; jj < kShrinkRowsPerCta; ++jj)
#pragma unroll
    for (int i = 0; i < kShrinkChunks; ++i) {
      const int k = tid * 8 + i * kStep;
      av[jj][i] = (lora && j0 + jj < R && k < K)
                      ? __ldg(reinterpret_cast<const uint4*>(Aad + (int64_t)(j0 + jj) * K + k))
                      : make_uint4(0, 0, 0, 0);
    }
  if (norm_w != nullptr) {
    __shared__ float ssq[kShrinkThreads / 32];
    uint4 wv[kShrinkChunks];
#pragma unroll
    for (int i = 0; i < kShrinkChunks; ++i) {
      const int k = tid * 8 + i * kStep;
      wv[i] = k < K ? *reinterpret_cast<const uint4*>(norm_w + k) : make_uint4(0, 0, 0, 0);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kShrinkChunks; ++i) {
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(u[q]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) ssq[wid] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kShrinkThreads / 32; ++w) tot += ssq[w];
    const float r = rsqrtf(tot / (float)K + eps);
#pragma unroll
    for (int i = 0; i < kShrinkChunks; ++i) {
      const int k = tid * 8 + i * kStep;
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
      const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv[i]);
      uint4 o;
      uint32_t* uo = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(u[q]);
        const float2 g = unpack_bf16x2(uw[q]);
        uo[q] = pack_bf16x2(f.x * r * g.x, f.y * r * g.y);
      }
      v[i] = o;
      if (k < K && xn != nullptr && blockIdx.y == 0) *reinterpret_cast<uint4*>(xn + (int64_t)t * xn_stride + k) = o;
    }
  }
  float acc[kShrinkRowsPerCta] = {};
#pragma unroll
  for (int i = 0; i < kShrinkChunks; ++i) {
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[i]);
#pragma unroll
    for (int jj = 0; jj < kShrinkRowsPerCta; ++jj) {
      const uint32_t* ua = reinterpret_cast<const uint32_t*>(&av[jj][i]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(u[q]);
        const float2 g = unpack_bf16x2(ua[q]);
        acc[jj] = fmaf(f.x, g.x, acc[jj]);
        acc[jj] = fmaf(f.y, g.y, acc[jj]);
      }
    }
  }
#pragma unroll
  for (int jj = 0; jj < kShrinkRowsPerCta; ++jj) {
    const float sv = warp_sum(acc[jj]);
    if (lane == 0) part[wid][jj] = sv;
  }
  __syncthreads();
  if (tid < kShrinkRowsPerCta && j0 + tid < R) {
    float sv = 0.f;
#pragma unroll
    for (int w = 0; w < kShrinkThreads / 32; ++w) sv += part[w][tid];
    down[(int64_t)t * down_stride + j0 + tid] = lora ? sv : 0.f;
  }
}

// ------------------------------------------------------------ merge weight
__global__ void lora_merge_weight_kernel(const bf16* __restrict__ w_in, bf16* __restrict__ w_out,
                                         const bf16* __restrict__ A, const bf16* __restrict__ B, int N, int K,
                                         int R, float scale, float sign, int mode) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t chunks = (int64_t)N * (K / 8);
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < chunks; c += (int64_t)gridDim.x * blockDim.x) {
    const int o = (int)(c / (K / 8));
    const int col = (int)(c % (K / 8)) * 8;
    float d[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = 0.f;
    for (int j = 0; j < R; ++j) {
      const float bj = bf2f(B[(int64_t)o * R + j]);
      uint4 av = *reinterpret_cast<const uint4*>(A + (int64_t)j * K + col);
      const uint32_t* ua = reinterpret_cast<const uint32_t*>(&av);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float2 f = unpack_bf16x2(ua[q]);
        d[2 * q] += bj * f.x;
        d[2 * q + 1] += bj * f.y;
      }
    }
    uint4 wv = *reinterpret_cast<const uint4*>(w_in + (int64_t)o * K + col);
    const uint32_t* uw = reinterpret_cast<const uint32_t*>(&wv);
    uint4 out;
    uint32_t* uo = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float2 wf = unpack_bf16x2(uw[q]);
      float r[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float wi = h ? wf.y : wf.x;
        const float dm = bfr(d[2 * q + h]);  // the bf16 matmul output B @ A
        if (mode == 0) {
          r[h] = wi + sign * bfr(dm * scale);
        } else {
          r[h] = wi + sign * scale * dm;
        }
      }
      uo[q] = pack_bf16x2(r[0], r[1]);
    }
    *reinterpret_cast<uint4*>(w_out + (int64_t)o * K + col) = out;
  }
}

}  // namespace pl

// =================================================================== host
PL_TRACE_READER(pl_trace_read_gemv)

namespace {
// Pipeline shape of linear_lora_kernel (pl_linear_set_tuning): ring depth,
// columns per 16-row stage, consumer warps, CTAs per SM.
int g_gemv_stages = 3;
int g_gemv_kc = 2048;
int g_gemv_consumers = 8;
int g_gemv_ctas_per_sm = 1;
int g_gemv_mode = 1;          // 0: by size, 1: TMA ring, 2: register-direct loads
int g_ldg_warps = 4;
int g_ldg_ctas_per_sm = 4;
int64_t g_auto_ldg_max_bytes = int64_t(64) << 20;  // mode 0: register-direct up to this many weight bytes
int64_t g_l2_prefetch_bytes = 0;  // register-direct variant: L2 prefetch budget per launch
}  // namespace

namespace {
// Checks the arguments of one fused GEMV projection and fills its argument
// block; *skip = true when there is nothing to compute.
int32_t gemv_args_from(const PlGemvPhase& q, pl::GemvArgs& a, bool* skip) {
  *skip = false;
  const void* x = q.x;
  const int64_t x_stride = q.x_stride;
  const int32_t num_tokens = q.num_tokens, k_in = q.k_in, prologue = q.prologue, n_out = q.n_out;
  const int32_t lora_rank = q.lora_rank, num_slices = q.num_slices, flags = q.flags;
  int32_t n_shrink = q.n_shrink;
  const bool down_from_x = (flags & PL_FLAG_DOWN_FROM_X) != 0;
  if (down_from_x) {  // shrink_a is the LoRA A stack [n_shrink adapters][lora_rank][k_in]
    if (q.lora_b == nullptr || q.shrink_a == nullptr || n_shrink < 1 || lora_rank <= 0 || num_slices > 1)
      return PL_ERR_INVALID_ARGUMENT;
    if (lora_rank > 64) return PL_ERR_UNSUPPORTED;
  }
  if (num_tokens == 0 || (n_out == 0 && (n_shrink == 0 || down_from_x))) {
    *skip = true;
    return PL_OK;
  }
  if (x == nullptr || q.w == nullptr || num_tokens < 0 || num_tokens > pl::kMaxTok || k_in <= 0 || n_out < 0 ||
      n_shrink < 0)
    return PL_ERR_INVALID_ARGUMENT;
  if (k_in % 16 != 0) return PL_ERR_UNSUPPORTED;
  if (n_out > 0 && q.y == nullptr) return PL_ERR_INVALID_ARGUMENT;
  if (!down_from_x && n_shrink > 0 && (q.shrink_a == nullptr || q.shrink_out == nullptr))
    return PL_ERR_INVALID_ARGUMENT;
  if (prologue == PL_PROLOGUE_RMSNORM && q.norm_w == nullptr) return PL_ERR_INVALID_ARGUMENT;
  if (prologue < 0 || prologue > 2) return PL_ERR_INVALID_ARGUMENT;
  if (q.lora_b != nullptr && ((q.lora_down == nullptr && !down_from_x) || lora_rank <= 0 || num_slices < 1 ||
                              num_slices > 4))
    return PL_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(q.w) & 15) || (x_stride % 8) ||
      (q.shrink_a != nullptr && (reinterpret_cast<uintptr_t>(q.shrink_a) & 15)) ||
      (q.norm_w != nullptr && (reinterpret_cast<uintptr_t>(q.norm_w) & 15)))
    return PL_ERR_INVALID_ARGUMENT;

  a = {};
  a.x = static_cast<const pl::bf16*>(x);
  a.x_stride = x_stride;
  a.T = num_tokens;
  a.K = k_in;
  a.prologue = prologue;
  a.norm_w = static_cast<const pl::bf16*>(q.norm_w);
  a.eps = q.norm_eps;
  a.w = static_cast<const pl::bf16*>(q.w);
  a.n_out = n_out;
  a.bias = static_cast<const pl::bf16*>(q.bias);
  a.lora_down = q.lora_down;
  a.down_stride = q.down_stride;
  a.lora_b = static_cast<const pl::bf16*>(q.lora_b);
  a.rank = lora_rank;
  a.lora_scale = q.lora_scale;
  a.num_slices = num_slices < 1 ? 1 : num_slices;
  for (int i = 0; i < 4; ++i) a.slice_end[i] = n_out;
  for (int i = 0; i < num_slices - 1 && i < 3; ++i) a.slice_end[i] = q.slice_end[i];
  a.tok_adapter = q.tok_adapter;
  a.residual = static_cast<const pl::bf16*>(q.residual);
  a.res_stride = q.res_stride;
  a.y = static_cast<pl::bf16*>(q.y);
  a.y_stride = q.y_stride;
  if (down_from_x) {
    a.pro_a = static_cast<const pl::bf16*>(q.shrink_a);
    a.pro_a_adapters = n_shrink;
    n_shrink = 0;  // no shrink rows: the down values stay in the kernel
  } else {
    a.shrink_a = static_cast<const pl::bf16*>(q.shrink_a);
    a.shrink_out = q.shrink_out;
    a.shrink_stride = q.shrink_stride;
  }
  a.n_shrink = n_shrink;
  a.early_weights = (flags & PL_FLAG_WEIGHTS_STATIC) ? 1 : 0;
  return PL_OK;
}

// Largest ring that fits: the tuned shape, then shallower / narrower stages.
bool gemv_ring_shape(int T, int k_max, int down_floats, int* stages_out, int* kc_out, int* smem_out) {
  int stages = g_gemv_stages, kc = g_gemv_kc;
  pl::GemvSmem L = pl::gemv_smem_layout(T, k_max, stages, kc, down_floats);
  while (L.total > 227 * 1024 && (stages > 2 || kc > 256)) {
    if (stages > 2) {
      --stages;
    } else {
      kc /= 2;
      stages = g_gemv_stages;
    }
    L = pl::gemv_smem_layout(T, k_max, stages, kc, down_floats);
  }
  if (L.total > 227 * 1024) return false;
  *stages_out = stages;
  *kc_out = kc;
  *smem_out = L.total;
  return true;
}
}  // namespace

namespace {
int32_t launch_gemv_phase(const PlGemvPhase& q, const PlGemvPrefetch* next, int32_t* status_dev, void* stream);
}  // namespace

extern "C" int32_t pl_linear_lora_expand_fused(const void* x, int64_t x_stride, int32_t num_tokens, int32_t k_in,
                                               int32_t prologue, const void* norm_w, float norm_eps, const void* w,
                                               int32_t n_out, const void* bias, const float* lora_down,
                                               int64_t down_stride, const void* lora_b, int32_t lora_rank,
                                               float lora_scale,
                                               const int32_t* slice_end, int32_t num_slices,
                                               const int32_t* tok_adapter, const void* residual, int64_t res_stride,
                                               void* y, int64_t y_stride, const void* shrink_a, int32_t n_shrink,
                                               float* shrink_out, int64_t shrink_stride, int32_t flags,
                                               int32_t* status_dev, void* stream) {
  PlGemvPhase q = {};
  q.x = x;
  q.x_stride = x_stride;
  q.num_tokens = num_tokens;
  q.k_in = k_in;
  q.prologue = prologue;
  q.norm_w = norm_w;
  q.norm_eps = norm_eps;
  q.w = w;
  q.n_out = n_out;
  q.bias = bias;
  q.lora_down = lora_down;
  q.down_stride = down_stride;
  q.lora_b = lora_b;
  q.lora_rank = lora_rank;
  q.lora_scale = lora_scale;
  q.num_slices = num_slices;
  if (num_slices > 4) return PL_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < num_slices - 1 && slice_end != nullptr; ++i) q.slice_end[i] = slice_end[i];
  q.tok_adapter = tok_adapter;
  q.residual = residual;
  q.res_stride = res_stride;
  q.y = y;
  q.y_stride = y_stride;
  q.shrink_a = shrink_a;
  q.n_shrink = n_shrink;
  q.shrink_out = shrink_out;
  q.shrink_stride = shrink_stride;
  q.flags = flags;
  if (num_slices > 1 && slice_end == nullptr) return PL_ERR_INVALID_ARGUMENT;
  return launch_gemv_phase(q, nullptr, status_dev, stream);
}

namespace {
int32_t launch_gemv_phase(const PlGemvPhase& q, const PlGemvPrefetch* next, int32_t* status_dev, void* stream) {
  pl::GemvArgs a;
  bool skip = false;
  int32_t st0 = gemv_args_from(q, a, &skip);
  if (st0 != PL_OK || skip) return st0;
  a.status = status_dev;
  const bool down_from_x = a.pro_a != nullptr;
  const int32_t num_tokens = q.num_tokens, k_in = q.k_in, n_out = q.n_out, lora_rank = q.lora_rank;
  const int32_t n_shrink = a.n_shrink;

  int sms = pl_host::sm_count();
  if (sms <= 0) sms = 148;
  const int64_t rows = (int64_t)n_out + n_shrink;
  const int64_t tiles = (rows + pl::kTileRows - 1) / pl::kTileRows;
  const bool ldg = !down_from_x && k_in % 32 == 0 &&
                   (g_gemv_mode == 2 || (g_gemv_mode == 0 && rows * k_in * 2 <= g_auto_ldg_max_bytes));
  if (ldg) {
    // register-direct variant: several CTAs per SM, tiles strided over the grid
    const pl::LdgSmem Ld = pl::ldg_smem_layout(num_tokens, k_in, g_ldg_warps);
    if (Ld.total > 227 * 1024) return PL_ERR_UNSUPPORTED;
    const int64_t cap = (int64_t)sms * g_ldg_ctas_per_sm;
    const int grid_l = (int)(tiles < cap ? tiles : cap);
    const int64_t tile_bytes = (int64_t)pl::kTileRows * k_in * 2;
    int64_t pf = g_l2_prefetch_bytes / ((int64_t)grid_l * tile_bytes);
    const int64_t per_cta = (tiles + grid_l - 1) / grid_l;
    a.prefetch_tiles = (int)(pf < per_cta ? pf : per_cta);
    if (g_ldg_warps == 8) {
      int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(pl::linear_ldg_kernel<8>), Ld.total);
      if (st != PL_OK) return st;
      return pl_host::launch_pdl(pl::linear_ldg_kernel<8>, dim3(grid_l), dim3(256), Ld.total, stream, a);
    }
    int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(pl::linear_ldg_kernel<4>), Ld.total);
    if (st != PL_OK) return st;
    return pl_host::launch_pdl(pl::linear_ldg_kernel<4>, dim3(grid_l), dim3(128), Ld.total, stream, a);
  }
  const int64_t max_ctas = (int64_t)sms * g_gemv_ctas_per_sm;
  const int grid = (int)(tiles < max_ctas ? tiles : max_ctas);
  int stages, kc, smem;
  const int down_floats = a.pro_a != nullptr ? num_tokens * lora_rank : 0;
  if (!gemv_ring_shape(num_tokens, k_in, down_floats, &stages, &kc, &smem)) return PL_ERR_UNSUPPORTED;
  a.stages = stages;
  a.kc = kc;
  if (next != nullptr && next->units > 0) {
    // the next launch's split: its grid and ring shape, as it will compute them
    const int64_t n_rows = (int64_t)next->n_out + next->n_shrink;
    const int64_t n_tiles = (n_rows + pl::kTileRows - 1) / pl::kTileRows;
    int n_stages, n_kc, n_smem;
    if (n_rows > 0 && gemv_ring_shape(next->num_tokens, next->k_in, 0, &n_stages, &n_kc, &n_smem)) {
      a.pf_w = static_cast<const pl::bf16*>(next->w);
      a.pf_shrink = static_cast<const pl::bf16*>(next->shrink_a);
      a.pf_rows_total = n_rows;
      a.pf_n_out = next->n_out;
      a.pf_k = next->k_in;
      a.pf_kc = n_kc;
      a.pf_units = next->units;
      a.pf_grid = (int)(n_tiles < max_ctas ? n_tiles : max_ctas);
    }
  }
  if (g_gemv_consumers == 8) {
    int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(pl::linear_lora_kernel<8>), smem);
    if (st != PL_OK) return st;
    return pl_host::launch_pdl(pl::linear_lora_kernel<8>, dim3(grid), dim3(32 * 9), smem, stream, a);
  }
  int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(pl::linear_lora_kernel<4>), smem);
  if (st != PL_OK) return st;
  return pl_host::launch_pdl(pl::linear_lora_kernel<4>, dim3(grid), dim3(32 * 5), smem, stream, a);
}

}  // namespace

extern "C" int32_t pl_linear_lora_phase(const PlGemvPhase* phase, const PlGemvPrefetch* next, int32_t* status_dev,
                                        void* stream) {
  if (phase == nullptr) return PL_ERR_INVALID_ARGUMENT;
  if (phase->num_slices > 4) return PL_ERR_INVALID_ARGUMENT;
  if (next != nullptr && next->units != 0) {
    if (next->units < 0 || next->units > 64 || next->w == nullptr || next->n_out < 0 || next->n_shrink < 0 ||
        (next->n_shrink > 0 && next->shrink_a == nullptr) || next->k_in <= 0 || next->num_tokens < 1 ||
        next->num_tokens > pl::kMaxTok || (reinterpret_cast<uintptr_t>(next->w) & 15) ||
        (reinterpret_cast<uintptr_t>(next->shrink_a) & 15))
      return PL_ERR_INVALID_ARGUMENT;
    if (next->k_in % 16) return PL_ERR_UNSUPPORTED;
  }
  return launch_gemv_phase(*phase, next, status_dev, stream);
}

extern "C" int32_t pl_linear_lora_chain(const PlGemvPhase* phases, int32_t num_phases, int32_t* grid_barrier,
                                        int32_t* status_dev, void* stream) {
  if (num_phases == 0) return PL_OK;
  if (phases == nullptr || num_phases < 0) return PL_ERR_INVALID_ARGUMENT;
  if (num_phases > pl::kMaxChainPhases) return PL_ERR_UNSUPPORTED;
  if (num_phases > 1 && (grid_barrier == nullptr || (reinterpret_cast<uintptr_t>(grid_barrier) & 3)))
    return PL_ERR_INVALID_ARGUMENT;
  pl::GemvChainArgs c = {};
  int n = 0, k_max = 0, down_max = 0, T = -1;
  for (int p = 0; p < num_phases; ++p) {
    const PlGemvPhase& q = phases[p];
    if (q.num_slices > 1 && q.num_slices <= 4) {
      for (int i = 0; i < q.num_slices - 1; ++i)
        if (q.slice_end[i] <= 0) return PL_ERR_INVALID_ARGUMENT;
    }
    bool skip = false;
    pl::GemvArgs a;
    const int32_t st = gemv_args_from(q, a, &skip);
    if (st != PL_OK) return st;
    if (skip) continue;
    if (T < 0) T = a.T;
    if (a.T != T) return PL_ERR_INVALID_ARGUMENT;  // one token count for the whole chain
    // lora_down is read through L1: it must not be the shrink output of an earlier phase
    for (int e = 0; e < n && a.lora_down != nullptr; ++e) {
      const pl::GemvArgs& b = c.ph[e];
      if (b.shrink_out != nullptr && a.lora_down >= b.shrink_out &&
          a.lora_down < b.shrink_out + (int64_t)(b.T - 1) * b.shrink_stride + b.n_shrink)
        return PL_ERR_UNSUPPORTED;
    }
    a.status = status_dev;
    a.coherent = 1;
    a.early_weights = 1;  // the producer streams every phase's weights without an upstream wait
    if (a.K > k_max) k_max = a.K;
    const int df = a.pro_a != nullptr ? a.T * a.rank : 0;
    if (df > down_max) down_max = df;
    c.ph[n++] = a;
  }
  if (n == 0) return PL_OK;
  int stages, kc, smem;
  if (!gemv_ring_shape(T, k_max, down_max, &stages, &kc, &smem)) return PL_ERR_UNSUPPORTED;
  for (int p = 0; p < n; ++p) {
    c.ph[p].stages = stages;
    c.ph[p].kc = kc;
  }
  c.num_phases = n;
  c.stages = stages;
  c.kc = kc;
  c.k_max = k_max;
  c.down_max = down_max;
  c.barrier = grid_barrier;
  c.status = status_dev;
  if (n > 1 && grid_barrier == nullptr) return PL_ERR_INVALID_ARGUMENT;
  // One CTA per SM: every CTA is resident at once (the grid barrier relies on it).
  int sms = pl_host::sm_count();
  if (sms <= 0) return PL_ERR_NO_DEVICE;
  int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(pl::linear_chain_kernel<8>), smem);
  if (st != PL_OK) return st;
  return pl_host::launch_pdl(pl::linear_chain_kernel<8>, dim3(sms), dim3(32 * 9), smem, stream, c);
}

extern "C" int32_t pl_linear_set_tuning(int32_t mode, int32_t stages, int32_t cols_per_stage,
                                        int32_t consumer_warps, int32_t ctas_per_sm) {
  if (mode == -1) {  // built-in defaults
    g_gemv_mode = 1;
    g_gemv_stages = 3;
    g_gemv_kc = 2048;
    g_gemv_consumers = 8;
    g_gemv_ctas_per_sm = 1;
    g_ldg_warps = 4;
    g_ldg_ctas_per_sm = 4;
    g_l2_prefetch_bytes = 0;
    return PL_OK;
  }
  if (mode < 0 || mode > 2 || stages < 2 || stages > 16 || cols_per_stage < 256 || cols_per_stage > 4096 ||
      cols_per_stage % 256 || (consumer_warps != 4 && consumer_warps != 8) || ctas_per_sm < 1 || ctas_per_sm > 16)
    return PL_ERR_INVALID_ARGUMENT;
  g_gemv_mode = mode;
  if (mode == 0) return PL_OK;
  if (mode == 2) {
    g_ldg_ctas_per_sm = ctas_per_sm;
    g_ldg_warps = consumer_warps;
    return PL_OK;
  }
  if (ctas_per_sm > 4) return PL_ERR_INVALID_ARGUMENT;
  g_gemv_stages = stages;
  g_gemv_kc = cols_per_stage;
  g_gemv_consumers = consumer_warps;
  g_gemv_ctas_per_sm = ctas_per_sm;
  return PL_OK;
}

extern "C" int32_t pl_linear_set_l2_prefetch(int64_t max_bytes) {
  if (max_bytes < 0 || max_bytes > (int64_t(1) << 30)) return PL_ERR_INVALID_ARGUMENT;
  g_l2_prefetch_bytes = max_bytes;
  return PL_OK;
}

extern "C" int32_t pl_lora_shrink_seg(const void* x, int64_t x_stride, const void* a, int32_t num_adapters,
                                      int32_t rank, int32_t in_features, const int32_t* seg_indptr,
                                      const int32_t* seg_adapter, int32_t num_segments, int32_t num_tokens,
                                      float* down, int64_t down_stride, void* stream) {
  if (num_tokens == 0 || num_segments == 0 || rank == 0) return PL_OK;
  if (x == nullptr || a == nullptr || seg_indptr == nullptr || seg_adapter == nullptr || down == nullptr ||
      rank < 0 || in_features <= 0 || num_segments < 0 || num_adapters <= 0 || num_segments > 65535)
    return PL_ERR_INVALID_ARGUMENT;
  if (in_features % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(a) & 15) ||
      (x_stride % 8))
    return PL_ERR_UNSUPPORTED;
  return pl_host::launch_pdl(pl::lora_shrink_kernel, dim3(rank, num_segments), dim3(256), 0, stream,
                             static_cast<const pl::bf16*>(x), x_stride, static_cast<const pl::bf16*>(a),
                             (int)num_adapters, (int)rank, (int)in_features, seg_indptr, seg_adapter, down,
                             down_stride);
}

extern "C" int32_t pl_lora_shrink_rows(const void* x, int64_t x_stride, int32_t num_tokens, int32_t k_in,
                                       const void* norm_w, float norm_eps, void* xn_out, int64_t xn_stride,
                                       const void* a, int32_t num_adapters, int32_t rank,
                                       const int32_t* tok_adapter, float* down, int64_t down_stride, void* stream) {
  if (num_tokens == 0 || rank == 0) return PL_OK;
  if (x == nullptr || a == nullptr || down == nullptr || num_tokens < 0 || k_in <= 0 || rank < 0 ||
      num_adapters <= 0 || num_tokens > 2147483647 / 2 || (xn_out != nullptr && norm_w == nullptr) ||
      down_stride < rank)
    return PL_ERR_INVALID_ARGUMENT;
  if (k_in % 8 || k_in > pl::kShrinkThreads * 8 * pl::kShrinkChunks || x_stride % 8 ||
      (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(a) & 15) ||
      (norm_w != nullptr && (reinterpret_cast<uintptr_t>(norm_w) & 15)) ||
      (xn_out != nullptr && ((reinterpret_cast<uintptr_t>(xn_out) & 15) || xn_stride % 8)))
    return PL_ERR_UNSUPPORTED;
  const int jb = (rank + pl::kShrinkRowsPerCta - 1) / pl::kShrinkRowsPerCta;
  if (jb > 65535) return PL_ERR_UNSUPPORTED;
  return pl_host::launch_pdl(pl::lora_shrink_rows_kernel, dim3(num_tokens, jb), dim3(pl::kShrinkThreads), 0,
                             stream, static_cast<const pl::bf16*>(x), x_stride, (int)k_in,
                             static_cast<const pl::bf16*>(norm_w), norm_eps, static_cast<pl::bf16*>(xn_out),
                             xn_stride, static_cast<const pl::bf16*>(a), (int)num_adapters, (int)rank, tok_adapter,
                             down, down_stride);
}

extern "C" int32_t pl_lora_merge_weight(const void* w_in, void* w_out, const void* a, const void* b, int32_t n_out,
                                        int32_t k_in, int32_t rank, float scale, int32_t sign, int32_t mode,
                                        void* stream) {
  if (n_out == 0 || k_in == 0) return PL_OK;
  if (w_in == nullptr || w_out == nullptr || a == nullptr || b == nullptr || n_out < 0 || k_in < 0 || rank <= 0 ||
      (sign != 1 && sign != -1) || (mode != 0 && mode != 1))
    return PL_ERR_INVALID_ARGUMENT;
  if (k_in % 8 != 0 || (reinterpret_cast<uintptr_t>(w_in) & 15) || (reinterpret_cast<uintptr_t>(w_out) & 15) ||
      (reinterpret_cast<uintptr_t>(a) & 15))
    return PL_ERR_UNSUPPORTED;
  int sms = pl_host::sm_count();
  if (sms <= 0) sms = 148;
  const int64_t chunks = (int64_t)n_out * (k_in / 8);
  int64_t blocks = (chunks + 255) / 256;
  if (blocks > 8LL * sms) blocks = 8LL * sms;
  return pl_host::launch_pdl(pl::lora_merge_weight_kernel, dim3((unsigned)blocks), dim3(256), 0, stream,
                             static_cast<const pl::bf16*>(w_in), static_cast<pl::bf16*>(w_out),
                             static_cast<const pl::bf16*>(a), static_cast<const pl::bf16*>(b), (int)n_out, (int)k_in,
                             (int)rank, scale, (float)sign, (int)mode);
}
