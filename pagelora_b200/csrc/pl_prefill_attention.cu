// Paged prefill attention (ragged, causal or not) on the 5th-generation
// tensor cores: the kernel behind pl_paged_prefill, replacing FlashInfer's
// BatchPrefillWithPagedKVCacheWrapper that the reference plans and runs in
// model/flashinfer/attention_backend.py:133-190 (pos_encoding_mode NONE, NHD
// layout, sm_scale = query_rescale / sqrt(D) on q / query_rescale).
//
// One CTA takes one (request, pair of query tiles, kv head).  A query tile
// is 128 tensor-core rows = TQ tokens x the `group` query heads that share
// the kv head (TQ = 128 / group), so every K/V tile is read once for 2 x 128
// rows.  The request's kv tokens are visited in tiles of 128 (128 / page_size
// pages) up to the last position the pair's queries may see.  Per CTA:
//   warp 0     TMA producer: K_0, V_0, K_1, V_1, ... through a 3-slot ring,
//              one lane per (page, 64-dim half) box, one instruction per
//              tile half; pages past the request's end load from an
//              out-of-range coordinate, which the copy fills with zeros;
//   warp 1     one lane issues tcgen05.mma in ping-pong order
//                S_A(0) S_B(0) | PV_A(0) S_A(1) PV_B(0) S_B(1) | PV_A(1) ...
//              (S_X = Q_X.K^T into tile X's TMEM score columns, PV_X = P_X.V
//              accumulated into its TMEM output columns, V an MN-major
//              operand), so each softmax group works while the tensor core
//              runs the other tile's products;
//   warps 2-5  softmax of tile A, warps 6-9 of tile B: one thread per tile
//              row stages the row's q, then per kv tile reads the row's
//              scores from TMEM, masks (causal / length), runs the online
//              softmax in the log2 domain and writes P (bf16) into the
//              tile's swizzled shared-memory P operand; at the end it
//              normalises O from TMEM and stores it.  Scores are
//              exponentiated against the running row maximum in one pass;
//              only a row whose maximum grows by more than 2^8 (and the
//              first tile) takes a max pass first and rescales O.
// Waits are bounded; on expiry the kernel records PL_ERR_TIMEOUT, lets its
// copies and tensor-core work drain (bounded) and returns.
#include "pl_common.cuh"

namespace pl {

constexpr int kPrefillThreads = 320;
constexpr int kPrefillM = 128;         // rows of one query tile
constexpr int kPrefillN = 128;         // kv tokens per tile
constexpr int kPrefillSlots = 3;       // K/V ring slots (one K or V tile each)
constexpr float kRescaleSlack = 8.0f;  // log2 growth of the row max tolerated before rescaling O

struct PrefillArgs {
  const bf16* q;
  int64_t q_stride_t, q_stride_h;
  const int32_t* qo_indptr;
  const int32_t* kv_indptr;
  const int32_t* kv_indices;
  const int32_t* kv_last;
  int64_t num_pages;
  int32_t batch, total_q, num_qo_heads, group, tq, page_size, causal;
  float scale_log2;
  bf16* out;
  int64_t out_stride_t, out_stride_h;
  float* lse;  // optional [total_q, Hq], natural log
  int32_t* status;
};

template <int D>
struct PrefillCfg {
  static constexpr int kChunks = D / 64;                   // 64-dim (128-byte) column chunks
  static constexpr int kChunkBytes = kPrefillM * 128;      // one chunk of a 128-row tile: 16 KB
  static constexpr int kQBytes = kChunks * kChunkBytes;    // one query tile
  static constexpr int kKVBytes = kChunks * kChunkBytes;   // K (or V) of 128 kv tokens
  static constexpr int kPBytes = 2 * kChunkBytes;          // P: 128 rows x 128 kv bf16
  static constexpr int kQOff = 0;                          // Q_A, Q_B
  static constexpr int kPOff = kQOff + 2 * kQBytes;        // P_A, P_B
  static constexpr int kSlotOff = kPOff + 2 * kPBytes;     // K/V ring
  static constexpr int kBarOff = kSlotOff + kPrefillSlots * kKVBytes;
  // full[3] empty[3] s[2] p[2] o[2] q[2] fin
  static constexpr int kNumBars = 2 * kPrefillSlots + 9;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;  // tmem slot, flags
  static constexpr int kSmemBytes = 1024 + kMiscOff + 64;
  static constexpr int kTmemCols = 512;                    // S_A 0, S_B 128, O_A 256, O_B 384
  static_assert(kSmemBytes <= 232448, "prefill tiles exceed the shared-memory limit");
};

// Byte offset of 16-byte unit `u` of row `r` in a 128B-swizzled K-major chunk.
__device__ __forceinline__ uint32_t pf_swz(int r, int u) { return r * 128 + ((u ^ (r & 7)) << 4); }

// 2^x on the multi-function unit (PTX ex2.approx, flush-to-zero); x = -inf gives 0.
__device__ __forceinline__ float pf_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
__global__ void __launch_bounds__(kPrefillThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap kv_map, const PrefillArgs a) {
  using C = PrefillCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* full = bars;                          // [3] ring slot landed
  uint64_t* empty = bars + kPrefillSlots;         // [3] ring slot free
  uint64_t* sready = bars + 2 * kPrefillSlots;    // [2] S_X in TMEM
  uint64_t* pready = sready + 2;                  // [2] P_X in shared memory (128 arrivals)
  uint64_t* odone = sready + 4;                   // [2] O_X += P_X.V finished
  uint64_t* qready = sready + 6;                  // [2] Q_X staged (128 arrivals)
  uint64_t* fin = sready + 8;                     // every tensor-core op of the CTA finished
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int32_t* flags = reinterpret_cast<volatile int32_t*>(smem + C::kMiscOff + 16);  // abort, issued, consumed

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int kvh = blockIdx.y;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPrefillSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&sready[x], 1);
      mbar_init(&pready[x], 128);
      mbar_init(&odone[x], 1);
      mbar_init(&qready[x], 128);
    }
    mbar_init(fin, 1);
    flags[0] = flags[1] = flags[2] = 0;
    fence_barrier_init();
  }
  if (threadIdx.x == 32) prefetch_tensormap(&kv_map);
  __syncthreads();
  pdl_launch_dependents();
  pdl_wait();  // q, the page table and the KV pages come from upstream kernels

  // ---- this CTA's (request, tile pair): heavier (later) pairs of a request first
  const int tq2 = 2 * a.tq;
  int req = -1, pair = 0, qo_begin = 0, qlen = 0;
  {
    int acc = 0;
    for (int b = 0; b < a.batch; ++b) {
      const int q0 = a.qo_indptr[b], q1 = a.qo_indptr[b + 1];
      const int n = q1 > q0 ? (q1 - q0 + tq2 - 1) / tq2 : 0;
      if ((int)blockIdx.x < acc + n) {
        req = b;
        pair = n - 1 - ((int)blockIdx.x - acc);
        qo_begin = q0;
        qlen = q1 - q0;
        break;
      }
      acc += n;
    }
  }
  if (blockIdx.x == 0 && kvh == 0 && threadIdx.x == 0) {
    if (a.qo_indptr[0] < 0 || a.qo_indptr[a.batch] > a.total_q) set_status(a.status, PL_ERR_INVALID_ARGUMENT);
  }
  if (req < 0) return;  // past the last pair: nothing allocated yet
  if (qo_begin < 0 || qo_begin + qlen > a.total_q) {
    if (threadIdx.x == 0) set_status(a.status, PL_ERR_INVALID_ARGUMENT);
    return;
  }
  const int PS = a.page_size;
  const int kv_begin = a.kv_indptr[req];
  const int n_pages = a.kv_indptr[req + 1] - kv_begin;
  int last = a.kv_last[req];
  last = last < 0 ? 0 : (last > PS ? PS : last);
  const int kv_len = n_pages > 0 ? (n_pages - 1) * PS + last : 0;
  const int t0 = pair * tq2;
  const int t1 = min(t0 + tq2, qlen);
  int n_vis = a.causal ? kv_len - qlen + t1 : kv_len;  // kv positions the pair's queries may see
  n_vis = n_vis < 0 ? 0 : (n_vis > kv_len ? kv_len : n_vis);
  const int ntiles = (n_vis + kPrefillN - 1) / kPrefillN;
  // The CTAs resident at one time mostly share a kv head and would walk the
  // same K/V tiles in lock-step, all hitting the same L2 lines; each starts
  // at its own tile instead (online softmax is order-free).
  const int rot = ntiles > 1 ? (int)(((unsigned)pair * 7u + (unsigned)kvh * 3u) % (unsigned)ntiles) : 0;
  auto tile_of = [&](int it) { return it + rot < ntiles ? it + rot : it + rot - ntiles; };

  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // item i: tile i / 2, K (even) or V (odd), ring slot i % 3
    const int ppt = kPrefillN / PS;       // pages per kv tile
    const int boxes = ppt * C::kChunks;   // <= 16 (host checks)
    const int p = lane / C::kChunks, hh = lane % C::kChunks;
    int i = 0;
    for (; i < 2 * ntiles; ++i) {
      const int s = i % kPrefillSlots;
      bool ok = true;
      if (i >= kPrefillSlots) ok = mbar_wait(&empty[s], ((i / kPrefillSlots) - 1) & 1);
      if (__any_sync(0xffffffffu, !ok || flags[0] != 0)) {  // one decision for the whole warp
        if (lane == 0 && !__all_sync(0xffffffffu, ok)) set_status(a.status, PL_ERR_TIMEOUT);
        flags[0] = 1;
        break;
      }
      if (lane == 0) mbar_arrive_expect_tx(&full[s], C::kKVBytes);
      __syncwarp();
      if (lane < boxes) {
        const int kv = i & 1, page_idx = tile_of(i >> 1) * ppt + p;
        int32_t coord = (int32_t)(2 * a.num_pages);  // out of range: the copy writes zeros
        if (page_idx < n_pages) {
          const int32_t pid = a.kv_indices[kv_begin + page_idx];
          if (pid >= 0 && (int64_t)pid < a.num_pages)
            coord = 2 * pid + kv;
          else
            set_status(a.status, PL_ERR_PAGE_OUT_OF_RANGE);
        }
        uint8_t* dst = smem + C::kSlotOff + s * C::kKVBytes + hh * C::kChunkBytes + p * PS * 128;
        tma_load_4d(dst, &kv_map, hh * 64, kvh, 0, coord, &full[s]);
      }
    }
    if (lane == 0) flags[1] = i;
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kPrefillM, kPrefillN);
      constexpr uint32_t idesc_o = umma_idesc_bf16(kPrefillM, D) | (1u << 16);  // B (V) MN-major
      int consumed = 0;  // ring items whose arrival was observed
      bool ok = ntiles == 0 || (mbar_wait(&qready[0], 0) && mbar_wait(&qready[1], 0));
      auto wait_item = [&](int item) -> bool {
        const bool r = mbar_wait(&full[item % kPrefillSlots], (item / kPrefillSlots) & 1) && !flags[0];
        if (r && item + 1 > consumed) consumed = item + 1;
        if (r) tc_fence_after();
        return r;
      };
      auto issue_s = [&](int x, int j) {  // S_X = Q_X . K_j^T
        const uint32_t qb = smem_u32(smem + C::kQOff + x * C::kQBytes);
        const uint32_t kb = smem_u32(smem + C::kSlotOff + ((2 * j) % kPrefillSlots) * C::kKVBytes);
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16(tmem + (uint32_t)(x * kPrefillN), umma_desc_k_sw128(qb + c * C::kChunkBytes + 32 * k),
                      umma_desc_k_sw128(kb + c * C::kChunkBytes + 32 * k), idesc_s, (c | k) ? 1u : 0u);
        umma_commit(&sready[x]);
      };
      auto issue_pv = [&](int x, int j) {  // O_X += P_X . V_j
        const uint32_t pb = smem_u32(smem + C::kPOff + x * C::kPBytes);
        const uint32_t vb = smem_u32(smem + C::kSlotOff + ((2 * j + 1) % kPrefillSlots) * C::kKVBytes);
#pragma unroll
        for (int kk = 0; kk < kPrefillN / 16; ++kk)
          umma_bf16(tmem + (uint32_t)(256 + x * 128), umma_desc_k_sw128(pb + (kk >> 2) * C::kChunkBytes + 32 * (kk & 3)),
                    umma_desc_mn_sw128(vb + kk * 16 * 128, C::kChunkBytes, 1024), idesc_o,
                    (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&odone[x]);
      };
      if (ok && ntiles > 0) {
        ok = wait_item(0);
        if (ok) {
          issue_s(0, 0);
          issue_s(1, 0);
          umma_commit(&empty[0]);  // K_0 read by both products
        }
      }
      for (int j = 0; ok && j < ntiles; ++j) {
        const bool more = j + 1 < ntiles;
        ok = mbar_wait(&pready[0], j & 1) && wait_item(2 * j + 1);
        if (!ok) break;
        tc_fence_after();
        issue_pv(0, j);
        if (more) {
          ok = wait_item(2 * j + 2);
          if (!ok) break;
          issue_s(0, j + 1);
        }
        ok = mbar_wait(&pready[1], j & 1) && !flags[0];
        if (!ok) break;
        tc_fence_after();
        issue_pv(1, j);
        umma_commit(&empty[(2 * j + 1) % kPrefillSlots]);  // V_j done
        if (more) {
          issue_s(1, j + 1);
          umma_commit(&empty[(2 * j + 2) % kPrefillSlots]);  // K_{j+1} done
        }
      }
      if (!ok) {
        set_status(a.status, PL_ERR_TIMEOUT);
        flags[0] = 1;
      }
      flags[2] = consumed;
      umma_commit(fin);  // arrives once everything issued above has finished
      if (!mbar_wait(fin, 0)) set_status(a.status, PL_ERR_TIMEOUT);
    }
  } else {
    // -------------------------------------------------- softmax / epilogue
    const int x = warp < 6 ? 0 : 1;  // query tile A (warps 2-5) or B (warps 6-9)
    const int quad = warp & 3;
    const int m = 32 * quad + lane;  // tile row == TMEM lane
    const int tok = t0 + x * a.tq + m / a.group;
    const int head = kvh * a.group + m % a.group;
    const bool row_ok = m < a.tq * a.group && tok < t1;
    const uint32_t row_tmem = tmem + ((uint32_t)(32 * quad) << 16);
    const uint32_t s_tmem = row_tmem + (uint32_t)(x * kPrefillN);
    const uint32_t o_tmem = row_tmem + (uint32_t)(256 + x * 128);

    // stage q (rows outside the tile are zero)
    {
      const bf16* src = a.q + (int64_t)(qo_begin + tok) * a.q_stride_t + (int64_t)head * a.q_stride_h;
      uint8_t* qs = smem + C::kQOff + x * C::kQBytes;
#pragma unroll
      for (int u = 0; u < D / 8; ++u) {
        const uint4 v = row_ok ? __ldg(reinterpret_cast<const uint4*>(src) + u) : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(qs + (u >> 3) * C::kChunkBytes + pf_swz(m, u & 7)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&qready[x]);
    }

    // last kv position this row may see (rows outside the tile see all)
    const int lim = (a.causal && row_ok) ? kv_len - qlen + tok : kv_len - 1;
    const float sl2 = a.scale_log2;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      ok = mbar_wait(&sready[x], j & 1);
      if (__any_sync(0xffffffffu, !ok || flags[0] != 0)) {  // tcgen05.ld below is warp-wide
        ok = false;
        break;
      }
      tc_fence_after();
      const int kv0 = tile_of(j) * kPrefillN;
      const bool masked = kv0 + kPrefillN - 1 > lim;  // some column of this row is masked
      // P_X and O_X are free once P_X(j-1).V_{j-1} has run (S_X(j) was issued
      // after it, so this wait returns at once)
      if (j >= 1) ok = mbar_wait(&odone[x], (j - 1) & 1);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint8_t* pt = smem + C::kPOff + x * C::kPBytes;
      // One pass against the running maximum; a row whose maximum grows by
      // more than 2^kRescaleSlack (and the first tile) takes the two-pass path.
      // Max and sum run as 8 independent chains each.
      bool two_pass = __any_sync(0xffffffffu, m_run == -INFINITY);
      if (!two_pass) {
        const float nb = -m_run;
        float sm[8], mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          sm[k] = 0.f;
          mx[k] = -INFINITY;
        }
#pragma unroll 1
        for (int h = 0; h < kPrefillN / 64; ++h) {
          float v[64];
          tmem_ld64(s_tmem + 64 * h, v);
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const int col = kv0 + 64 * h + i;
            float p0 = pf_exp2(fmaf(v[i], sl2, nb));
            float p1 = pf_exp2(fmaf(v[i + 1], sl2, nb));
            float s0 = v[i], s1 = v[i + 1];
            if (masked) {
              const bool k0 = col <= lim, k1 = col + 1 <= lim;
              p0 = k0 ? p0 : 0.f;
              p1 = k1 ? p1 : 0.f;
              s0 = k0 ? s0 : -INFINITY;
              s1 = k1 ? s1 : -INFINITY;
            }
            mx[(i >> 1) & 7] = fmaxf(mx[(i >> 1) & 7], fmaxf(s0, s1));
            sm[(i >> 1) & 7] += p0 + p1;
            pk[i / 2] = pack_bf16x2(p0, p1);
          }
          uint8_t* chunk = pt + h * C::kChunkBytes;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(chunk + pf_swz(m, u)) =
                make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
        const float vmax =
            fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        two_pass = __any_sync(0xffffffffu, vmax * sl2 > m_run + kRescaleSlack);
        if (!two_pass) l_run += ((sm[0] + sm[1]) + (sm[2] + sm[3])) + ((sm[4] + sm[5]) + (sm[6] + sm[7]));
      }
      if (two_pass) {
        // pass 1: row maximum of the masked scores
        float mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
#pragma unroll 1
        for (int h = 0; h < kPrefillN / 64; ++h) {
          float v[64];
          tmem_ld64(s_tmem + 64 * h, v);
          if (masked) {
#pragma unroll
            for (int i = 0; i < 64; ++i) mx[i & 7] = fmaxf(mx[i & 7], kv0 + 64 * h + i <= lim ? v[i] : -INFINITY);
          } else {
#pragma unroll
            for (int i = 0; i < 64; ++i) mx[i & 7] = fmaxf(mx[i & 7], v[i]);
          }
        }
        float tmax =
            fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        tmax *= sl2;  // sl2 > 0: the max commutes with the scaling
        const float m_new = fmaxf(m_run, tmax);
        const bool rescale = m_run != -INFINITY && m_new > m_run + kRescaleSlack;
        const float m_use = (m_run == -INFINITY || rescale) ? m_new : m_run;
        if (__any_sync(0xffffffffu, rescale)) {
          const float alpha = rescale ? pf_exp2(m_run - m_use) : 1.f;
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            float v[16];
            tmem_ld16(o_tmem + 16 * c, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] *= alpha;
            tmem_st16_wait(o_tmem + 16 * c, v);
          }
          l_run *= alpha;
        }
        m_run = m_use;
        // pass 2: P = exp2(s * scale - m), row sum, bf16 P into the swizzled tile
        const float nb = m_use == -INFINITY ? 0.f : -m_use;
        float sm[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) sm[k] = 0.f;
#pragma unroll 1
        for (int h = 0; h < kPrefillN / 64; ++h) {
          float v[64];
          tmem_ld64(s_tmem + 64 * h, v);
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const int col = kv0 + 64 * h + i;
            float p0 = pf_exp2(fmaf(v[i], sl2, nb));
            float p1 = pf_exp2(fmaf(v[i + 1], sl2, nb));
            if (masked) {
              p0 = col <= lim ? p0 : 0.f;
              p1 = col + 1 <= lim ? p1 : 0.f;
            }
            sm[(i >> 1) & 7] += p0 + p1;
            pk[i / 2] = pack_bf16x2(p0, p1);
          }
          uint8_t* chunk = pt + h * C::kChunkBytes;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(chunk + pf_swz(m, u)) =
                make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
        l_run += ((sm[0] + sm[1]) + (sm[2] + sm[3])) + ((sm[4] + sm[5]) + (sm[6] + sm[7]));
      }
      // Slots past the request's last token in its last page hold whatever
      // the pool had there (0 * NaN is NaN): tile A's threads clear those V
      // rows (P_A.V_j runs first, after this tile's arrival).
      const int tail0 = kv_len - kv0, tail1 = min(kPrefillN, n_pages * PS - kv0);
      if (x == 0 && tail0 >= 0 && tail0 < tail1) {
        const int item = 2 * j + 1;
        if (mbar_wait(&full[item % kPrefillSlots], (item / kPrefillSlots) & 1)) {
          uint8_t* vt = smem + C::kSlotOff + (item % kPrefillSlots) * C::kKVBytes;
          const int units = (tail1 - tail0) * C::kChunks * 8;
          for (int idx = m; idx < units; idx += 128) {
            const int r = tail0 + idx / (C::kChunks * 8), hh = (idx / 8) % C::kChunks, u = idx % 8;
            *reinterpret_cast<uint4*>(vt + hh * C::kChunkBytes + r * 128 + u * 16) = make_uint4(0, 0, 0, 0);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&pready[x]);
    }
    if (!ok) {
      set_status(a.status, PL_ERR_TIMEOUT);
      flags[0] = 1;
    }
    // ---- epilogue: O / l  (ok is warp-uniform here)
    bool have_o = false;
    if (ok && ntiles > 0) {
      have_o = __all_sync(0xffffffffu, mbar_wait(&odone[x], (ntiles - 1) & 1));
      if (!have_o) {
        set_status(a.status, PL_ERR_TIMEOUT);
        flags[0] = 1;
      }
    }
    tc_fence_after();
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    bf16* dst = a.out + (int64_t)(qo_begin + tok) * a.out_stride_t + (int64_t)head * a.out_stride_h;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      float v[32];
      if (have_o) {
        tmem_ld32(o_tmem + 32 * c, v);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      if (row_ok && !flags[0]) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) pk[i / 2] = pack_bf16x2(v[i] * inv, v[i + 1] * inv);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          reinterpret_cast<uint4*>(dst + 32 * c)[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
      }
    }
    if (a.lse != nullptr && row_ok && !flags[0])
      a.lse[(int64_t)(qo_begin + tok) * a.num_qo_heads + head] =
          l_run > 0.f ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
  }

  // ------------------------------------------------------------ teardown
  __syncthreads();
  if (threadIdx.x == 0) {
    // copies issued but never consumed (abort only) must land before exit
    const int issued = flags[1], consumed = flags[2];
    for (int i = consumed; i < issued; ++i) (void)mbar_wait(&full[i % kPrefillSlots], (i / kPrefillSlots) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace pl

// =================================================================== host
namespace {

template <int D>
int32_t launch_prefill(const CUtensorMap& map, const pl::PrefillArgs& a, int grid_x, int hkv, void* stream) {
  using C = pl::PrefillCfg<D>;
  auto kern = pl::paged_prefill_kernel<D>;
  int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes);
  if (st != PL_OK) return st;
  return pl_host::launch_pdl(kern, dim3(grid_x, hkv), dim3(pl::kPrefillThreads), C::kSmemBytes, stream, map, a);
}

}  // namespace

extern "C" int32_t pl_paged_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* kv_cache,
                                    int64_t num_pages, const int32_t* qo_indptr, const int32_t* kv_indptr,
                                    const int32_t* kv_indices, const int32_t* kv_last_page_len, int32_t batch,
                                    int32_t total_q, int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
                                    int32_t page_size, float sm_scale, int32_t causal, void* out,
                                    int64_t out_stride_t, int64_t out_stride_h, float* out_lse, int32_t* status_dev,
                                    void* stream) {
  if (q == nullptr || kv_cache == nullptr || qo_indptr == nullptr || kv_indptr == nullptr || kv_indices == nullptr ||
      kv_last_page_len == nullptr || out == nullptr || batch < 0 || total_q < 0 || num_pages <= 0 ||
      num_kv_heads <= 0 || num_qo_heads <= 0 || num_qo_heads % num_kv_heads != 0)
    return PL_ERR_INVALID_ARGUMENT;
  const int group = num_qo_heads / num_kv_heads;
  if (group > pl::kPrefillM || (head_dim != 64 && head_dim != 128) ||
      (page_size != 16 && page_size != 32 && page_size != 64 && page_size != 128))
    return PL_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(kv_cache) & 15) != 0 || (reinterpret_cast<uintptr_t>(q) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(out) & 15) != 0 || (q_stride_t % 8) != 0 || (q_stride_h % 8) != 0 ||
      (out_stride_t % 8) != 0 || (out_stride_h % 8) != 0)
    return PL_ERR_INVALID_ARGUMENT;
  if (batch == 0 || total_q == 0) return PL_OK;

  CUtensorMap map;
  int32_t st = pl_host::kv_tensor_map(kv_cache, num_pages, num_kv_heads, head_dim, page_size, &map);
  if (st != PL_OK) return st;

  pl::PrefillArgs a;
  a.q = static_cast<const pl::bf16*>(q);
  a.q_stride_t = q_stride_t;
  a.q_stride_h = q_stride_h;
  a.qo_indptr = qo_indptr;
  a.kv_indptr = kv_indptr;
  a.kv_indices = kv_indices;
  a.kv_last = kv_last_page_len;
  a.num_pages = num_pages;
  a.batch = batch;
  a.total_q = total_q;
  a.num_qo_heads = num_qo_heads;
  a.group = group;
  a.tq = pl::kPrefillM / group;
  a.page_size = page_size;
  a.causal = causal ? 1 : 0;
  a.scale_log2 = sm_scale * pl::kLog2e;
  a.out = static_cast<pl::bf16*>(out);
  a.out_stride_t = out_stride_t;
  a.out_stride_h = out_stride_h;
  a.lse = out_lse;
  a.status = status_dev;
  // every request contributes ceil(len / 2tq) <= len / 2tq + 1 tile pairs
  const int64_t grid_x = ((int64_t)total_q + 2 * a.tq - 1) / (2 * a.tq) + batch;
  if (grid_x > 0x7FFFFFFF) return PL_ERR_INVALID_ARGUMENT;
  if (head_dim == 128) return launch_prefill<128>(map, a, (int)grid_x, num_kv_heads, stream);
  return launch_prefill<64>(map, a, (int)grid_x, num_kv_heads, stream);
}
