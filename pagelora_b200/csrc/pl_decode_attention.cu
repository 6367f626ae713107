// Paged-KV GQA decode attention for sm_100a, plus the split-KV LSE merge.
//
// One CTA per (row, kv head, kv split).  All `group` query heads that share
// the kv head sit in one CTA, so each KV page is read from HBM exactly once.
// Warp 0 is the producer: one lane per (page, K/V, 64-dim half) box issues
// TMA tile loads (128B-swizzled) for 8 pages per instruction into a ring of
// shared-memory stages, each guarded by a full/empty mbarrier pair, with the
// page ids read one batch ahead.  Warps 1..kConsumerWarps are consumers:
// stage s always belongs to consumer warp s % kConsumerWarps, which takes its
// pages in order (one waiter per full barrier, never a phase ahead), and runs
// Q.K^T and P.V on the tensor cores (mma.sync m16n8k16, fp32 accumulate;
// query heads are the M rows, only `group` of 16 used) with an online
// softmax in the log2 domain.  The consumer warps' states are combined
// through shared memory.  With several splits, the splits of a (row, kv
// head) form one thread-block cluster when the plan says so: every CTA
// pushes its (O, LSE) chunks into the reducing CTA's shared memory over
// DSMEM and each CTA reduces its own chunks after one cluster barrier;
// otherwise the partial states go to the workspace and the last CTA to
// arrive (atomic ticket, no spin) merges them.  Either way split-KV needs no
// second launch.  The fused form (pl_paged_decode_qkv) computes the rotated
// q heads from the packed projection row, and appends the new token's K/V,
// inside the same launch (pl_qkv_head.cuh).
//
// Semantics follow model/flashinfer/attention_backend.py:97,120-131:
// O = softmax((q/16) . K^T * 16/sqrt(D)) . V = softmax(q.K^T * sm_scale) . V
// over the pages indices[indptr[b] .. indptr[b+1]) of the NHD pool
// [P, 2, page_size, Hkv, D]; the last page holds last_page_len[b] tokens.
#include <mutex>
#include <vector>

#include "pl_qkv_head.cuh"

namespace pl {

// Consumer warps: 7 when a split's pages fit the ring in one lap (several
// splits of a short context: two pages at most per warp), 6 for long splits
// (where the 16-stage ring's ownership is as even at 6 and the extra warp
// measured slower).
template <int NCW>
constexpr int decode_threads() { return 32 * (1 + NCW); }

struct DecodeArgs {
  const bf16* q;
  int64_t q_stride_b, q_stride_h;
  const int32_t* indptr;
  const int32_t* indices;
  const int32_t* last_page_len;
  int64_t num_pages;
  int32_t num_qo_heads, num_kv_heads, group;
  float scale_log2;  // sm_scale * log2(e)
  int32_t num_splits;
  // Row folding (shared page lists): blockIdx.z is a page-table row shared by
  // `fold` consecutive query rows; tile row m is query row z*fold + m/group,
  // head kvh*group + m%group.  Rows >= rows_real are padding.
  int32_t fold;
  int32_t rows_real;
  int32_t cluster;      // 1: the splits of a (row, kv head) form one cluster and merge through DSMEM
  // Fused q/k/v: q is computed from the projection row (qh) instead of read
  // from `q`; the CTA that holds the row's last page appends the new token's
  // K/V at (slot_page, slot_off) and uses them directly in this step.
  int32_t fused;
  QkvHeadArgs qh;
  const int32_t* slot_page;
  const int32_t* slot_off;
  bf16* cache_w;        // the pool (writable) for the append
  bf16* q_out;          // nullable: the rotated q is also written here [B, Hq, D]
  bf16* out;
  float* out_f32;       // when set, O is written here in fp32 instead of `out`
  int64_t o_stride_b, o_stride_h;
  float* out_lse;       // natural log, nullable
  int32_t* counters;    // [batch * Hkv], zero between calls
  float* partial_o;     // [batch, Hq, splits, D]
  float* partial_lse;   // [batch, Hq, splits] (log2 domain)
  int32_t* status;
  // nullable: a prior state per (query row, head) -- O fp32 [rows][Hq][D],
  // LSE [rows][Hq] (natural log) -- merged into the bf16 output with the
  // arithmetic of merge_states_strided_kernel over [prior, this launch]
  const float* prior_o;
  const float* prior_lse;
};

template <int D, int PS, int NCW>
struct DecodeCfg {
  static constexpr int kConsumerWarps = NCW;
  static constexpr int kHalves = D / 64;              // 64-dim (128 B) boxes per tile
  static constexpr int kHalfBytes = PS * 128;         // one box: PS rows x 128 B
  static constexpr int kTileBytes = kHalves * kHalfBytes;  // K (or V) of one page/head
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kBoxesPerPage = 2 * kHalves;            // K and V, per 64-dim half
  static constexpr int kPagesPerBatch = 32 / kBoxesPerPage;    // pages per producer instruction
  // Two producer batches in flight, at most 128 KB of stages.
  static constexpr int kStages = (2 * kPagesPerBatch * kStageBytes <= 131072) ? 2 * kPagesPerBatch
                                                                              : 131072 / kStageBytes;
  static constexpr int kQRowBytes = D * 2 + 16;       // padded rows: conflict-free ldmatrix
  static constexpr int kNT = PS / 8;                  // score n-tiles per page
  static constexpr int kDT = D / 8;                   // output n-tiles
  // shared-memory carve-up (offsets from a 1024-aligned base)
  static constexpr int kStageOff = 0;
  static constexpr int kQOff = kStages * kStageBytes;
  static constexpr int kMLOff = kQOff + 16 * kQRowBytes;                 // [warps][16] m, l
  static constexpr int kBarOff = kMLOff + 2 * kConsumerWarps * 16 * 4;   // full[], empty[]
  static constexpr int kNtokOff = kBarOff + 2 * kStages * 8;
  static constexpr int kFlagOff = kNtokOff + kStages * 4;
  // Cluster merge: what the other splits push here (this CTA reduces the
  // float4 chunks j = split + S*i): O chunks [i][split] and LSE [split][row].
  static constexpr int kClOff = (kFlagOff + 16 + 15) & ~15;
  static constexpr int kClChunks = 16 * D / 4 + 16;                     // upper bound of i*S + s
  static constexpr int kClLseOff = kClOff + kClChunks * 16;
  static constexpr int kNewKvOff = kClLseOff + 16 * 16 * 4;             // fused: new K, V rows (bf16)
  static constexpr int kSmemBytes = kNewKvOff + 2 * D * 2 + 1024;      // + alignment slack
  static constexpr int kScratchRow = D + 4;                             // padded: conflict-free writes
  static_assert(kConsumerWarps * 16 * kScratchRow * 4 <= kStages * kStageBytes, "merge scratch must fit the stage ring");
  static_assert(kStages >= kPagesPerBatch, "one producer batch must map to distinct stages");
  static_assert(kStages >= kConsumerWarps, "every consumer warp owns at least one stage");
};

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a 128B-swizzled box.
__device__ __forceinline__ uint32_t swz128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

template <int D, int PS, int NCW>
__global__ void __launch_bounds__(decode_threads<NCW>()) paged_decode_kernel(const __grid_constant__ CUtensorMap kv_map,
                                                                              const DecodeArgs args) {
  using C = DecodeCfg<D, PS, NCW>;
  constexpr int kConsumerWarps = NCW;
  constexpr int kDecodeThreads = decode_threads<NCW>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty_bar = full_bar + C::kStages;
  int32_t* stage_ntok = reinterpret_cast<int32_t*>(smem + C::kNtokOff);
  volatile int32_t* flags = reinterpret_cast<volatile int32_t*>(smem + C::kFlagOff);  // [0]=abort [1]=is_last
  float* ml = reinterpret_cast<float*>(smem + C::kMLOff);                            // m[w][16], l[w][16]

  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int group = args.group;
  const int mrows = group * args.fold;  // tile rows in use (<= 16)
  auto row_of = [&](int m) { return (int)blockIdx.z * args.fold + m / group; };
  auto head_of = [&](int m) { return kvh * group + m % group; };
  // This launch's normalised output chunk v (LSE lse_nat, natural log)
  // merged with the prior state of (orow, ohead): merge_states_strided's
  // expressions over the states [prior, this], so the bf16 result equals the
  // separate merge launch's.
  auto with_prior = [&](int orow, int ohead, int d, float4 v, float lse_nat) -> float4 {
    const int64_t rh = (int64_t)orow * args.num_qo_heads + ohead;
    const float l0 = args.prior_lse[rh], l1 = lse_nat;
    float M = -INFINITY;
    M = fmaxf(M, l0);
    M = fmaxf(M, l1);
    float L = 0.f;
    if (M != -INFINITY) {
      L += expf(l0 - M);
      L += expf(l1 - M);
    }
    const float4 p = *reinterpret_cast<const float4*>(args.prior_o + rh * D + d);
    const float pv[4] = {p.x, p.y, p.z, p.w}, tv[4] = {v.x, v.y, v.z, v.w};
    float r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float acc = 0.f;
      if (M != -INFINITY) {
        acc += expf(l0 - M) * pv[i];
        acc += expf(l1 - M) * tv[i];
      }
      r[i] = L > 0.f ? acc / L : 0.f;
    }
    return make_float4(r[0], r[1], r[2], r[3]);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    flags[0] = 0;
    flags[1] = 0;
    fence_barrier_init();
  }
  if (threadIdx.x == 32) prefetch_tensormap(&kv_map);
  if (threadIdx.x == 0 && kvh == 0) PL_TRACE_POINT(0);
  __syncthreads();
  // Cluster merge: announce that this CTA runs (the others push into its
  // shared memory after their matching wait).
  if (args.cluster) cluster_arrive_relaxed();

  pdl_launch_dependents();
  if (args.fused && warp >= 1) {
    // static operands of this CTA's q heads (and of the K/V heads, which one
    // CTA of the row will need) into L2 while the upstream grid finishes
    const int cw = warp - 1;
    for (int r = cw; r < group; r += kConsumerWarps) qkv_head_prefetch<D>(args.qh, kvh * group + r, lane);
    const int kw = (cw + kConsumerWarps - group % kConsumerWarps) % kConsumerWarps;  // 0: K warp, 1: V warp
    if (kw < 2) qkv_head_prefetch<D>(args.qh, args.num_qo_heads + kw * args.num_kv_heads + kvh, lane);
  }
  pdl_wait();  // q, the page table and the freshly appended KV come from upstream kernels
  if (threadIdx.x == 0 && kvh == 0) PL_TRACE_POINT(1);

  const int32_t row_begin = args.indptr[b];
  const int32_t n_pages = args.indptr[b + 1] - row_begin;
  const int32_t pps = (n_pages + args.num_splits - 1) / args.num_splits;
  const int32_t p0 = min(split * pps, n_pages);
  const int32_t p1 = min(p0 + pps, n_pages);
  const int32_t n = p1 - p0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // A TMA instruction costs ~0.3 us of issue time however many lanes issue
    // it, so the warp loads a batch of pages per instruction: one lane per
    // (page, K/V, 64-dim half) box.
    if (n > 0) {
      int32_t last_len = args.last_page_len[b];
      last_len = last_len < 0 ? 0 : (last_len > PS ? PS : last_len);
      const int box = lane % C::kBoxesPerPage;
      const bool lane_used = lane < C::kBoxesPerPage * C::kPagesPerBatch;
      // Page ids are read one batch ahead, so the index load's latency hides
      // behind the wait for free stages instead of delaying the copies.
      int32_t pid_next = (lane_used && lane / C::kBoxesPerPage < n)
                             ? args.indices[row_begin + p0 + lane / C::kBoxesPerPage]
                             : 0;
      int issued = 0;
      for (int i0 = 0; i0 < n; i0 += C::kPagesPerBatch) {
        const int i = i0 + lane / C::kBoxesPerPage;
        const bool active = lane_used && i < n;
        const int s = i % C::kStages;
        const int32_t pid_here = pid_next;
        pid_next = (lane_used && i + C::kPagesPerBatch < n)
                       ? args.indices[row_begin + p0 + i + C::kPagesPerBatch]
                       : 0;
        bool ok = true;
        if (active && i >= C::kStages) ok = mbar_wait(&empty_bar[s], ((i / C::kStages) - 1) & 1);
        if (!__all_sync(0xffffffffu, ok)) {
          if (lane == 0) set_status(args.status, PL_ERR_TIMEOUT);
          flags[0] = 1;
          break;
        }
        const int32_t page_idx = p0 + i;
        const int32_t pid = active ? pid_here : 0;
        const int32_t ntok = (page_idx == n_pages - 1) ? last_len : PS;
        const bool valid = active && pid >= 0 && static_cast<int64_t>(pid) < args.num_pages && ntok > 0;
        if (active && box == 0) {
          if (!valid) {
            if (ntok != 0) set_status(args.status, PL_ERR_PAGE_OUT_OF_RANGE);
            stage_ntok[s] = 0;
            mbar_arrive(&full_bar[s]);  // nothing to load: consumers skip the page
          } else {
            stage_ntok[s] = ntok;
            mbar_arrive_expect_tx(&full_bar[s], C::kStageBytes);
          }
        }
        __syncwarp();
        if (lane == 0 && i0 == 0 && kvh == 0) PL_TRACE_POINT(2);
        if (valid) {
          const int kv = box / C::kHalves, hh = box % C::kHalves;
          uint8_t* dst = smem + C::kStageOff + s * C::kStageBytes + kv * C::kTileBytes + hh * C::kHalfBytes;
          tma_load_4d(dst, &kv_map, hh * 64, kvh, 0, 2 * pid + kv, &full_bar[s]);
        }
        issued = min(n, i0 + C::kPagesPerBatch);
      }
      if (flags[0] && lane == 0) {
        // Abort: wait (bounded) for the loads still in flight before the CTA exits.
        for (int i = issued - C::kStages < 0 ? 0 : issued - C::kStages; i < issued; ++i)
          (void)mbar_wait(&full_bar[i % C::kStages], (i / C::kStages) & 1);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int cw = warp - 1;        // consumer warp 0..3
    const int ctid = threadIdx.x - 32;
    const int g = lane >> 2;        // fragment row (query head within group)
    const int t = lane & 3;

    // Stage q rows (zero-padded to 16) into shared memory.
    uint8_t* qs = smem + C::kQOff;
    bool appender = false;  // fused: this CTA holds the row's last page, where the new token goes
    int new_off = 0;
    if (!args.fused) {
      constexpr int kChunksPerRow = D / 8;
      for (int idx = ctid; idx < 16 * kChunksPerRow; idx += 32 * kConsumerWarps) {
        const int r = idx / kChunksPerRow, c = idx % kChunksPerRow;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < mrows && row_of(r) < args.rows_real) {
          const bf16* src =
              args.q + (int64_t)row_of(r) * args.q_stride_b + (int64_t)head_of(r) * args.q_stride_h + c * 8;
          v = *reinterpret_cast<const uint4*>(src);
        }
        *reinterpret_cast<uint4*>(qs + r * C::kQRowBytes + c * 16) = v;
      }
    } else {
      constexpr int E = D / 32;
      constexpr int kChunksPerRow = D / 8;
      for (int idx = ctid; idx < (16 - group) * kChunksPerRow; idx += 32 * kConsumerWarps) {
        const int r = group + idx / kChunksPerRow, c = idx % kChunksPerRow;
        *reinterpret_cast<uint4*>(qs + r * C::kQRowBytes + c * 16) = make_uint4(0, 0, 0, 0);
      }
      // q heads of this group: normalised and rotated, one warp per head
      for (int r = cw; r < group; r += kConsumerWarps) {
        float v[E];
        qkv_head_transform<D>(args.qh, b, kvh * group + r, lane, v);
        bf16* dst = reinterpret_cast<bf16*>(qs + r * C::kQRowBytes) + lane * E;
#pragma unroll
        for (int e = 0; e < E; ++e) dst[e] = f2bf(v[e]);
        if (args.q_out != nullptr && split == 0) {
          bf16* g = args.q_out + ((int64_t)b * args.num_qo_heads + kvh * group + r) * D + lane * E;
#pragma unroll
          for (int e = 0; e < E; ++e) g[e] = f2bf(v[e]);
        }
      }
      // The new token lands in the row's last page: the CTA holding that
      // page computes its K/V, appends them and keeps them for this step.
      if (n > 0 && p1 == n_pages) {
        const int32_t last_pid = args.indices[row_begin + n_pages - 1];
        const int32_t llen = args.last_page_len[b];
        const int32_t spid = args.slot_page[b], soff = args.slot_off[b];
        appender = spid == last_pid && soff == llen - 1 && soff >= 0 && soff < PS && spid >= 0 &&
                   static_cast<int64_t>(spid) < args.num_pages;
        new_off = soff;
        // K and V go to the warps after the q heads' (idle ones when group < 5)
        const int kw = (cw + kConsumerWarps - group % kConsumerWarps) % kConsumerWarps;
        if (appender && kw < 2) {
          float v[E];
          qkv_head_transform<D>(args.qh, b, args.num_qo_heads + kw * args.num_kv_heads + kvh, lane, v);
          bf16* sm = reinterpret_cast<bf16*>(smem + C::kNewKvOff) + kw * D + lane * E;
          bf16* g = args.cache_w + ((((int64_t)spid * 2 + kw) * PS + soff) * args.num_kv_heads + kvh) * D + lane * E;
#pragma unroll
          for (int e = 0; e < E; ++e) {
            sm[e] = f2bf(v[e]);
            g[e] = f2bf(v[e]);
          }
        }
      }
    }
    named_barrier(1, 32 * kConsumerWarps);
    if (ctid == 0 && kvh == 0) PL_TRACE_POINT(9);
    // Every CTA of the cluster has started (the merge pushes into their
    // shared memory): waited for here, while the first pages are in flight,
    // rather than at the merge.
    if (args.cluster) cluster_wait();

    uint32_t qa[D / 16][4];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int r = (lane & 7) + 8 * ((lane >> 3) & 1);
      const int col = kk * 16 + 8 * (lane >> 4);
      ldsm_x4(smem_u32(qs + r * C::kQRowBytes + col * 2), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
    }

    float o[C::kDT][4];
#pragma unroll
    for (int j = 0; j < C::kDT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const float sl2 = args.scale_log2;

    // Stage s is always consumed by warp s % kConsumerWarps, in page order, so
    // each full barrier has one waiter that never runs a phase ahead.  (Dealt
    // round-robin across the ring's laps, a warp could reach page i while the
    // copy of page i - kStages into the same stage is still in flight: a
    // parity wait cannot tell that phase's successor from its predecessor and
    // would return at once on the old contents.)
    auto next_page = [&](int i) {
      return (i % C::kStages) + kConsumerWarps < C::kStages ? i + kConsumerWarps
                                                            : (i / C::kStages + 1) * C::kStages + cw;
    };
    for (int i = cw; i < n; i = next_page(i)) {
      const int s = i % C::kStages;
      if (!mbar_wait(&full_bar[s], (i / C::kStages) & 1)) {
        set_status(args.status, PL_ERR_TIMEOUT);
        flags[0] = 1;
        break;
      }
      if (flags[0]) break;
      if (i == 0 && lane == 0 && kvh == 0) PL_TRACE_POINT(3);
      if (appender && i == n - 1) {
        // The copy of the last page may predate the append: put the new
        // token's K and V rows into the staged tiles (16-byte chunks).
        constexpr int kRowChunks = D / 8;
        if (lane < 2 * kRowChunks) {
          const int kv = lane / kRowChunks, c = lane % kRowChunks;
          uint8_t* tile = smem + C::kStageOff + s * C::kStageBytes + kv * C::kTileBytes;
          *reinterpret_cast<uint4*>(tile + (c / 8) * C::kHalfBytes + swz128(new_off, c % 8)) =
              *reinterpret_cast<const uint4*>(smem + C::kNewKvOff + kv * D * 2 + c * 16);
        }
        __syncwarp();
      }
      const int ntok = stage_ntok[s];
      if (ntok > 0 && ntok < PS) {
        // Slots past the last token hold whatever the pool had there (the
        // reference allocates it uninitialised): their p is 0, but 0 * NaN
        // is NaN, so clear those V rows of the staged page.
        constexpr int kRowUnits = 8 * C::kHalves;
        uint8_t* vt = smem + C::kStageOff + s * C::kStageBytes + C::kTileBytes;
        for (int idx = lane; idx < (PS - ntok) * kRowUnits; idx += 32) {
          const int r = ntok + idx / kRowUnits, hh = (idx % kRowUnits) / 8, c = idx % 8;
          *reinterpret_cast<uint4*>(vt + hh * C::kHalfBytes + r * 128 + c * 16) = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      if (ntok > 0) {
        const uint8_t* kbase = smem + C::kStageOff + s * C::kStageBytes;
        const uint8_t* vbase = kbase + C::kTileBytes;
        // ---- S = Q . K^T  (16 x PS)
        float sc[C::kNT][4];
#pragma unroll
        for (int j = 0; j < C::kNT; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
          for (int jp = 0; jp < C::kNT / 2; ++jp) {
            const int m = lane >> 3;
            const int tok = jp * 16 + (m >> 1) * 8 + (lane & 7);
            const int gc = 2 * kk + (m & 1);
            const uint32_t addr = smem_u32(kbase + (gc >> 3) * C::kHalfBytes + swz128(tok, gc & 7));
            uint32_t kb[4];
            ldsm_x4(addr, kb[0], kb[1], kb[2], kb[3]);
            mma_bf16_16816(sc[2 * jp + 0], qa[kk], &kb[0]);
            mma_bf16_16816(sc[2 * jp + 1], qa[kk], &kb[2]);
          }
        }
        // ---- online softmax (rows g and g+8), log2 domain
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < C::kNT; ++j) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int tok = 8 * j + 2 * t + c;
            const bool valid = tok < ntok;
            sc[j][c] = valid ? sc[j][c] * sl2 : -INFINITY;
            sc[j][2 + c] = valid ? sc[j][2 + c] * sl2 : -INFINITY;
            mx0 = fmaxf(mx0, sc[j][c]);
            mx1 = fmaxf(mx1, sc[j][2 + c]);
          }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);
        m0 = mn0;
        m1 = mn1;
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int j = 0; j < C::kNT; ++j) {
          sc[j][0] = exp2f(sc[j][0] - mn0);
          sc[j][1] = exp2f(sc[j][1] - mn0);
          sc[j][2] = exp2f(sc[j][2] - mn1);
          sc[j][3] = exp2f(sc[j][3] - mn1);
          ps0 += sc[j][0] + sc[j][1];
          ps1 += sc[j][2] + sc[j][3];
        }
        l0 = l0 * a0 + ps0;
        l1 = l1 * a1 + ps1;
#pragma unroll
        for (int j = 0; j < C::kDT; ++j) {
          o[j][0] *= a0;
          o[j][1] *= a0;
          o[j][2] *= a1;
          o[j][3] *= a1;
        }
        // ---- O += P . V
#pragma unroll
        for (int kt = 0; kt < PS / 16; ++kt) {
          uint32_t pa[4];
          pa[0] = pack_bf16x2(sc[2 * kt][0], sc[2 * kt][1]);
          pa[1] = pack_bf16x2(sc[2 * kt][2], sc[2 * kt][3]);
          pa[2] = pack_bf16x2(sc[2 * kt + 1][0], sc[2 * kt + 1][1]);
          pa[3] = pack_bf16x2(sc[2 * kt + 1][2], sc[2 * kt + 1][3]);
#pragma unroll
          for (int dc = 0; dc < C::kDT; dc += 2) {
            const int m = lane >> 3;
            const int tok = kt * 16 + (m & 1) * 8 + (lane & 7);
            const int gc = dc + (m >> 1);
            const uint32_t addr = smem_u32(vbase + (gc >> 3) * C::kHalfBytes + swz128(tok, gc & 7));
            uint32_t vb[4];
            ldsm_x4_trans(addr, vb[0], vb[1], vb[2], vb[3]);
            mma_bf16_16816(o[dc], pa, &vb[0]);
            mma_bf16_16816(o[dc + 1], pa, &vb[2]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[s]);
    }

    // ---- merge the consumer warps' states (scratch aliases the drained stage ring)
    if (lane == 0 && kvh == 0) PL_TRACE_MAX(4);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    named_barrier(1, 32 * kConsumerWarps);  // every warp is done reading its stages
    if (ctid == 0 && kvh == 0) PL_TRACE_POINT(7);
    float* scratch = reinterpret_cast<float*>(smem + C::kStageOff);  // [warp][16][kScratchRow]
    float* mw = ml;                                                   // [warp][16]
    float* lw = ml + kConsumerWarps * 16;
    {
      constexpr int SR = C::kScratchRow;
      float* ow = scratch + cw * 16 * SR;
#pragma unroll
      for (int j = 0; j < C::kDT; ++j) {
        const int d = 8 * j + 2 * t;
        *reinterpret_cast<float2*>(ow + g * SR + d) = make_float2(o[j][0], o[j][1]);
        *reinterpret_cast<float2*>(ow + (g + 8) * SR + d) = make_float2(o[j][2], o[j][3]);
      }
      if (t == 0) {
        mw[cw * 16 + g] = m0;
        mw[cw * 16 + g + 8] = m1;
        lw[cw * 16 + g] = l0;
        lw[cw * 16 + g + 8] = l1;
      }
    }
    named_barrier(1, 32 * kConsumerWarps);
    if (ctid == 0 && kvh == 0) PL_TRACE_POINT(8);

    const bool single = args.num_splits == 1;
    // One float4 chunk (row r, columns d..d+3) per thread and pass: combine
    // the consumer warps' states, then write the output (one split), push
    // the chunk to the CTA of the cluster that reduces it, or leave it in
    // the workspace for the last CTA to arrive.
    for (int idx = ctid; idx < mrows * (D / 4); idx += 32 * kConsumerWarps) {
      const int r = idx / (D / 4), d = 4 * (idx % (D / 4));
      const int orow = row_of(r), ohead = head_of(r);
      const bool live = orow < args.rows_real;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mw[w * 16 + r]);
      float L = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float wt = exp2f(mw[w * 16 + r] - M);
          const float4 sv = *reinterpret_cast<const float4*>(scratch + (w * 16 + r) * C::kScratchRow + d);
          L += wt * lw[w * 16 + r];
          acc.x += wt * sv.x;
          acc.y += wt * sv.y;
          acc.z += wt * sv.z;
          acc.w += wt * sv.w;
        }
      }
      const float il = (L > 0.f) ? 1.f / L : 0.f;
      const float4 val = make_float4(acc.x * il, acc.y * il, acc.z * il, acc.w * il);
      const float lse2 = (L > 0.f) ? M + log2f(L) : -INFINITY;
      if (single) {
        if (live) {
          const int64_t oi = (int64_t)orow * args.o_stride_b + (int64_t)ohead * args.o_stride_h + d;
          if (args.out_f32 != nullptr) {
            *reinterpret_cast<float4*>(args.out_f32 + oi) = val;
          } else {
            const float4 w = args.prior_o != nullptr ? with_prior(orow, ohead, d, val, lse2 * kLn2) : val;
            reinterpret_cast<uint2*>(args.out + oi)[0] = make_uint2(pack_bf16x2(w.x, w.y), pack_bf16x2(w.z, w.w));
          }
          if (args.out_lse != nullptr && d == 0)
            args.out_lse[(int64_t)orow * args.num_qo_heads + ohead] = lse2 * kLn2;
        }
      } else if (args.cluster) {
        const int S = args.num_splits;
        const uint32_t dst = (uint32_t)(idx % S);  // reducer CTA of this chunk
        dsmem_st_f32x4(dsmem_map(smem_u32(smem + C::kClOff) + ((idx / S) * S + split) * 16, dst), val);
        if (d == 0) {
          const uint32_t lse_at = smem_u32(smem + C::kClLseOff) + (split * 16 + r) * 4;
          for (int c = 0; c < S; ++c) dsmem_st_f32(dsmem_map(lse_at, c), lse2);  // every reducer needs it
        }
      } else if (live) {
        const int64_t rowid = (int64_t)orow * args.num_qo_heads + ohead;
        *reinterpret_cast<float4*>(args.partial_o + (rowid * args.num_splits + split) * D + d) = val;
        if (d == 0) args.partial_lse[rowid * args.num_splits + split] = lse2;
      }
    }
    if (ctid == 0 && kvh == 0) PL_TRACE_POINT(10);
    if (!single && !args.cluster) {
      __threadfence();
      named_barrier(1, 32 * kConsumerWarps);
      if (ctid == 0) {
        const int32_t ticket = atomicAdd(&args.counters[b * args.num_kv_heads + kvh], 1);
        flags[1] = (ticket == args.num_splits - 1) ? 1 : 0;
      }
      named_barrier(1, 32 * kConsumerWarps);
      if (ctid == 0 && kvh == 0) PL_TRACE_POINT(5);
      if (flags[1]) {
        // Last CTA of this (row, kv head): merge the S partial states.  The
        // split weights are computed once per query head into shared memory,
        // then every thread reduces float4 columns with independent loads.
        __threadfence();
        const int S = args.num_splits;
        float* wts = scratch;              // [mrows][S] weights, then [mrows] 1/L
        float* inv_l = scratch + mrows * S;
        for (int idx = ctid; idx < mrows * S; idx += 32 * kConsumerWarps) {
          const int m = idx / S;
          wts[idx] = row_of(m) < args.rows_real
                         ? __ldcg(args.partial_lse + ((int64_t)row_of(m) * args.num_qo_heads + head_of(m)) * S +
                                  idx % S)
                         : -INFINITY;
        }
        named_barrier(1, 32 * kConsumerWarps);
        if (ctid < mrows) {
          float M = -INFINITY;
          for (int s = 0; s < S; ++s) M = fmaxf(M, wts[ctid * S + s]);
          float L = 0.f;
          for (int s = 0; s < S; ++s) {
            const float wt = (M == -INFINITY) ? 0.f : exp2f(wts[ctid * S + s] - M);
            wts[ctid * S + s] = wt;
            L += wt;
          }
          inv_l[ctid] = L > 0.f ? 1.f / L : 0.f;
          inv_l[mrows + ctid] = (L > 0.f) ? (M + log2f(L)) * kLn2 : -INFINITY;  // for a prior-state merge
          if (args.out_lse != nullptr && row_of(ctid) < args.rows_real)
            args.out_lse[(int64_t)row_of(ctid) * args.num_qo_heads + head_of(ctid)] =
                (L > 0.f) ? (M + log2f(L)) * kLn2 : -INFINITY;
        }
        named_barrier(1, 32 * kConsumerWarps);
        for (int idx = ctid; idx < mrows * (D / 4); idx += 32 * kConsumerWarps) {
          const int r = idx / (D / 4), d = 4 * (idx % (D / 4));
          if (row_of(r) >= args.rows_real) continue;
          const int64_t rowid = (int64_t)row_of(r) * args.num_qo_heads + head_of(r);
          const float4* src = reinterpret_cast<const float4*>(args.partial_o + (rowid * S) * D + d);
          const float* wr = wts + r * S;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
          for (int s = 0; s < S; ++s) {
            const float wt = wr[s];
            const float4 o = __ldcg(src + (int64_t)s * (D / 4));
            acc.x += wt * o.x;
            acc.y += wt * o.y;
            acc.z += wt * o.z;
            acc.w += wt * o.w;
          }
          const float il = inv_l[r];
          const int64_t oi = (int64_t)row_of(r) * args.o_stride_b + (int64_t)head_of(r) * args.o_stride_h + d;
          if (args.out_f32 != nullptr) {
            *reinterpret_cast<float4*>(args.out_f32 + oi) = make_float4(acc.x * il, acc.y * il, acc.z * il, acc.w * il);
          } else {
            float4 w = make_float4(acc.x * il, acc.y * il, acc.z * il, acc.w * il);
            if (args.prior_o != nullptr) w = with_prior(row_of(r), head_of(r), d, w, inv_l[mrows + r]);
            reinterpret_cast<uint2*>(args.out + oi)[0] = make_uint2(pack_bf16x2(w.x, w.y), pack_bf16x2(w.z, w.w));
          }
        }
        if (ctid == 0) args.counters[b * args.num_kv_heads + kvh] = 0;
        if (ctid == 0 && kvh == 0) PL_TRACE_POINT(6);
      }
    }
  }

  if (args.cluster) {
    // The splits of this (row, kv head) are the CTAs of one cluster (rank =
    // split).  Every CTA has pushed its chunk j to CTA j % S and its LSE to
    // all CTAs (remote stores, made visible by the barrier); each CTA then
    // reduces its chunks from its own shared memory.  Nothing is read
    // remotely, so no CTA waits for another one after the barrier.
    __syncwarp();
    if (warp == 0) cluster_wait();  // the producer warp's half of the start barrier
    if (threadIdx.x == 32 && kvh == 0) PL_TRACE_POINT(11);
    cluster_sync_all();
    if (threadIdx.x == 32 && kvh == 0) PL_TRACE_POINT(12);
    const int S = args.num_splits;
    const float4* recv = reinterpret_cast<const float4*>(smem + C::kClOff);
    const float* recv_lse = reinterpret_cast<const float*>(smem + C::kClLseOff);
    for (int i = threadIdx.x; i * S + split < mrows * (D / 4); i += kDecodeThreads) {
      const int j = i * S + split;  // chunk reduced here
      const int r = j / (D / 4), d = 4 * (j % (D / 4));
      if (row_of(r) >= args.rows_real) continue;
      float M = -INFINITY;
      for (int s = 0; s < S; ++s) M = fmaxf(M, recv_lse[s * 16 + r]);
      float L = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (M != -INFINITY) {
        for (int s = 0; s < S; ++s) {
          const float l = recv_lse[s * 16 + r];
          const float w = l == -INFINITY ? 0.f : exp2f(l - M);
          const float4 o = recv[i * S + s];
          L += w;
          acc.x += w * o.x;
          acc.y += w * o.y;
          acc.z += w * o.z;
          acc.w += w * o.w;
        }
      }
      if (i == 0 && threadIdx.x == 0 && kvh == 0) {
        asm volatile("" ::"f"(acc.x));
        PL_TRACE_POINT(14);
      }
      const float il = L > 0.f ? 1.f / L : 0.f;
      const int64_t oi = (int64_t)row_of(r) * args.o_stride_b + (int64_t)head_of(r) * args.o_stride_h + d;
      if (args.out_f32 != nullptr) {
        *reinterpret_cast<float4*>(args.out_f32 + oi) = make_float4(acc.x * il, acc.y * il, acc.z * il, acc.w * il);
      } else {
        float4 w = make_float4(acc.x * il, acc.y * il, acc.z * il, acc.w * il);
        if (args.prior_o != nullptr)
          w = with_prior(row_of(r), head_of(r), d, w, L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY);
        reinterpret_cast<uint2*>(args.out + oi)[0] = make_uint2(pack_bf16x2(w.x, w.y), pack_bf16x2(w.z, w.w));
      }
      if (args.out_lse != nullptr && d == 0)
        args.out_lse[(int64_t)row_of(r) * args.num_qo_heads + head_of(r)] =
            L > 0.f ? (M + log2f(L)) * kLn2 : -INFINITY;
    }
    if (threadIdx.x == 0 && kvh == 0) PL_TRACE_POINT(15);
  }
}

// ---------------------------------------------------------------- LSE merge
__global__ void merge_states_kernel(const float* __restrict__ v, const float* __restrict__ lse, int num_rows,
                                    int num_states, int head_dim, bf16* __restrict__ out, int64_t out_stride,
                                    float* __restrict__ out_lse) {
  pdl_wait();
  const int row = blockIdx.x;
  if (row >= num_rows) return;
  const float* l = lse + (int64_t)row * num_states;
  float M = -INFINITY;
  for (int s = 0; s < num_states; ++s) M = fmaxf(M, l[s]);
  float L = 0.f;
  if (M != -INFINITY)
    for (int s = 0; s < num_states; ++s) L += expf(l[s] - M);
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float acc = 0.f;
    if (M != -INFINITY)
      for (int s = 0; s < num_states; ++s) acc += expf(l[s] - M) * v[((int64_t)row * num_states + s) * head_dim + d];
    out[(int64_t)row * out_stride + d] = f2bf(L > 0.f ? acc / L : 0.f);
  }
  if (out_lse != nullptr && threadIdx.x == 0) out_lse[row] = L > 0.f ? M + logf(L) : -INFINITY;
}

// Same merge over partial states laid out with arbitrary row / state strides
// (e.g. [states][rows][D] as gathered from several GPUs).
__global__ void merge_states_strided_kernel(const float* __restrict__ v, int64_t v_row_stride, int64_t v_state_stride,
                                            const float* __restrict__ lse, int64_t lse_row_stride,
                                            int64_t lse_state_stride, int num_rows, int num_states, int head_dim,
                                            bf16* __restrict__ out, int64_t out_stride, float* __restrict__ out_lse) {
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  if (row >= num_rows) return;
  const float* l = lse + (int64_t)row * lse_row_stride;
  float M = -INFINITY;
  for (int s = 0; s < num_states; ++s) M = fmaxf(M, l[s * lse_state_stride]);
  float L = 0.f;
  if (M != -INFINITY)
    for (int s = 0; s < num_states; ++s) L += expf(l[s * lse_state_stride] - M);
  const float* vr = v + (int64_t)row * v_row_stride;
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float acc = 0.f;
    if (M != -INFINITY)
      for (int s = 0; s < num_states; ++s) acc += expf(l[s * lse_state_stride] - M) * vr[s * v_state_stride + d];
    out[(int64_t)row * out_stride + d] = f2bf(L > 0.f ? acc / L : 0.f);
  }
  if (out_lse != nullptr && threadIdx.x == 0) out_lse[row] = L > 0.f ? M + logf(L) : -INFINITY;
}

}  // namespace pl

// =================================================================== host
PL_TRACE_READER(pl_trace_read_attn)

namespace {

struct MapKey {
  const void* ptr;
  int64_t pages;
  int32_t hkv, d, ps, dev;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && pages == o.pages && hkv == o.hkv && d == o.d && ps == o.ps && dev == o.dev;
  }
};

constexpr int kMapCache = 128;
struct MapCache {
  std::mutex mu;
  MapKey key[kMapCache];
  CUtensorMap map[kMapCache];
  int used = 0, next = 0;
};
MapCache g_maps;

}  // namespace

namespace pl_host {
// Tensor map over one layer's pool viewed as [2*P][PS][Hkv][D] (innermost last):
// dims (inner->outer) {D, Hkv, PS, 2P}, box {64, 1, PS, 1}, 128B swizzle.
int32_t kv_tensor_map(const void* cache, int64_t pages, int hkv, int d, int ps, CUtensorMap* out) {
  int dev = 0;
  cudaGetDevice(&dev);
  MapKey k{cache, pages, hkv, d, ps, dev};
  std::lock_guard<std::mutex> lock(g_maps.mu);
  for (int i = 0; i < g_maps.used; ++i)
    if (g_maps.key[i] == k) {
      *out = g_maps.map[i];
      return PL_OK;
    }
  pl_host::EncodeTiledFn enc = pl_host::encode_tiled_fn();
  if (enc == nullptr) return PL_ERR_CUDA;
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)hkv, (cuuint64_t)ps, (cuuint64_t)(2 * pages)};
  cuuint64_t strides[3] = {(cuuint64_t)d * 2, (cuuint64_t)hkv * d * 2, (cuuint64_t)ps * hkv * d * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)ps, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMap m;
  CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(cache), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return PL_ERR_INVALID_ARGUMENT;
  int slot;
  if (g_maps.used < kMapCache) {
    slot = g_maps.used++;
  } else {
    slot = g_maps.next;
    g_maps.next = (g_maps.next + 1) % kMapCache;
  }
  g_maps.key[slot] = k;
  g_maps.map[slot] = m;
  *out = m;
  return PL_OK;
}
}  // namespace pl_host

namespace {

int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

int64_t decode_workspace_bytes(int batch, int hq, int hkv, int d, int splits) {
  if (splits <= 1) return align256((int64_t)batch * hkv * 4);
  return align256((int64_t)batch * hkv * 4) + align256((int64_t)batch * hq * splits * d * 4) +
         align256((int64_t)batch * hq * splits * 4);
}

// Consumer warps of a launch with `splits` splits (see decode_threads).
constexpr int consumer_warps_for(int splits) { return splits >= 3 ? 7 : 6; }

template <int D, int PS, int NCW>
int32_t launch_decode_ncw(const CUtensorMap& map, const pl::DecodeArgs& a, int batch, int hkv, int splits,
                          void* stream) {
  using C = pl::DecodeCfg<D, PS, NCW>;
  auto kern = pl::paged_decode_kernel<D, PS, NCW>;
  constexpr int threads = pl::decode_threads<NCW>();
  int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes);
  if (st != PL_OK) return st;
  if (a.cluster)
    return pl_host::launch_pdl_cluster(kern, dim3(splits, hkv, batch), dim3(threads), C::kSmemBytes, stream, splits,
                                       map, a);
  return pl_host::launch_pdl(kern, dim3(splits, hkv, batch), dim3(threads), C::kSmemBytes, stream, map, a);
}

template <int D, int PS>
int32_t launch_decode(const CUtensorMap& map, const pl::DecodeArgs& a, int batch, int hkv, int splits, void* stream) {
  if (consumer_warps_for(splits) == 7) return launch_decode_ncw<D, PS, 7>(map, a, batch, hkv, splits, stream);
  return launch_decode_ncw<D, PS, 6>(map, a, batch, hkv, splits, stream);
}

// Split merge through a thread-block cluster (the splits of one (row, kv
// head) as one cluster of up to 16 CTAs) when every cluster of the launch
// can be resident at once; answers are cached per kernel, size and device.
bool g_cluster_merge = true;
constexpr int kMaxClusterSplits = 16;

struct ClusterFit {
  const void* kernel;
  int dev, splits, active;
};
std::mutex g_fit_mu;
std::vector<ClusterFit> g_fits;

template <int D, int PS, int NCW>
int cluster_capacity_ncw(int splits) {
  using C = pl::DecodeCfg<D, PS, NCW>;
  auto kern = pl::paged_decode_kernel<D, PS, NCW>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  {
    std::lock_guard<std::mutex> lock(g_fit_mu);
    for (const auto& f : g_fits)
      if (f.kernel == reinterpret_cast<const void*>(kern) && f.dev == dev && f.splits == splits) return f.active;
  }
  int active = 0;
  if (pl_host::ensure_smem_attr(reinterpret_cast<const void*>(kern), C::kSmemBytes) == PL_OK &&
      (splits <= 8 ||
       cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess)) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, 1, 1);
    cfg.blockDim = dim3(pl::decode_threads<NCW>());
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) != cudaSuccess) active = 0;
  }
  cudaGetLastError();  // a refused query leaves no sticky error
  std::lock_guard<std::mutex> lock(g_fit_mu);
  g_fits.push_back({reinterpret_cast<const void*>(kern), dev, splits, active});
  return active;
}

template <int D, int PS>
int cluster_capacity(int splits) {
  if (consumer_warps_for(splits) == 7) return cluster_capacity_ncw<D, PS, 7>(splits);
  return cluster_capacity_ncw<D, PS, 6>(splits);
}

int cluster_capacity_for(int head_dim, int page_size, int splits) {
  if (head_dim == 128 && page_size == 16) return cluster_capacity<128, 16>(splits);
  if (head_dim == 128 && page_size == 32) return cluster_capacity<128, 32>(splits);
  if (head_dim == 64 && page_size == 16) return cluster_capacity<64, 16>(splits);
  if (head_dim == 64 && page_size == 32) return cluster_capacity<64, 32>(splits);
  return 0;
}

bool use_cluster_merge(int head_dim, int page_size, int splits, int64_t clusters) {
  return g_cluster_merge && splits >= 2 && splits <= kMaxClusterSplits &&
         (int64_t)cluster_capacity_for(head_dim, page_size, splits) >= clusters;
}

}  // namespace

extern "C" int32_t pl_decode_plan(int32_t batch, int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
                                  int32_t page_size, int64_t total_pages, int32_t max_splits,
                                  pl_decode_plan_t* plan_out) {
  if (plan_out == nullptr || batch < 0 || num_kv_heads <= 0 || num_qo_heads % num_kv_heads != 0 || head_dim <= 0 ||
      page_size <= 0 || total_pages < 0)
    return PL_ERR_INVALID_ARGUMENT;
  int sms = pl_host::sm_count();
  if (sms <= 0) sms = 148;
  const int64_t base = (int64_t)batch * num_kv_heads;
  int splits = 1;
  if (base > 0) {
    // One wave of CTAs, one per SM; each split keeps >= 4 pages so the
    // merge (proportional to the split count) stays small next to the scan.
    const int64_t target = sms;
    const int64_t avg_pages = (total_pages + batch - 1) / (batch > 0 ? batch : 1);
    int64_t by_fill = target / base;  // never more CTAs than SMs: the ring needs a whole SM
    int64_t by_len = avg_pages / 4;
    int64_t s = by_fill < by_len ? by_fill : by_len;
    if (s > 64) s = 64;
    if (max_splits > 0 && s > max_splits) s = max_splits;
    // Fewer splits are worth a cluster merge (no round trip through global
    // memory, no arrival ticket): take the largest split count whose clusters
    // all fit on the device at once (measured on B200: 10 at 8 clusters of
    // 137 KB CTAs, where 16-CTA clusters fit only 7 at a time).
    if (s >= 2 && g_cluster_merge) {
      for (int64_t c = s < kMaxClusterSplits ? s : kMaxClusterSplits; c >= 2; --c)
        if (use_cluster_merge(head_dim, page_size, (int)c, base)) {
          s = c;
          break;
        }
    }
    splits = s < 1 ? 1 : static_cast<int>(s);
  }
  plan_out->num_splits = splits;
  plan_out->ctas = static_cast<int32_t>(base * splits);
  plan_out->workspace_bytes = decode_workspace_bytes(batch, num_qo_heads, num_kv_heads, head_dim, splits);
  return PL_OK;
}

namespace {
int32_t paged_decode_impl(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* kv_cache,
                          int64_t num_pages, const int32_t* indptr, const int32_t* indices,
                          const int32_t* last_page_len, int32_t batch, int32_t num_qo_heads, int32_t num_kv_heads,
                          int32_t head_dim, int32_t page_size, float sm_scale, int32_t num_splits, void* out,
                          bool out_is_f32, int64_t o_stride_b, int64_t o_stride_h, float* out_lse, void* workspace,
                          int64_t workspace_bytes, int32_t* status_dev, void* stream,
                          const pl::QkvHeadArgs* fused = nullptr, const int32_t* slot_page = nullptr,
                          const int32_t* slot_off = nullptr, void* q_out = nullptr, int fold = 1,
                          int64_t counter_bytes = 0, const float* prior_o = nullptr,
                          const float* prior_lse = nullptr) {
  if (batch == 0) return PL_OK;
  if ((prior_o == nullptr) != (prior_lse == nullptr) ||
      (prior_o != nullptr && (out_is_f32 || (reinterpret_cast<uintptr_t>(prior_o) & 15))))
    return PL_ERR_INVALID_ARGUMENT;
  if (fused != nullptr) {  // q comes from the projection row: validate that instead
    if (fused->qkv == nullptr || fused->positions == nullptr || slot_page == nullptr || slot_off == nullptr ||
        (fused->down != nullptr && fused->lora_b != nullptr && fused->rank <= 0) ||
        fused->Hq != num_qo_heads || fused->Hkv != num_kv_heads)
      return PL_ERR_INVALID_ARGUMENT;
    q = kv_cache;  // any 16-byte aligned pointer: the q checks below do not apply
    q_stride_b = q_stride_h = 0;
  }
  if (q == nullptr || kv_cache == nullptr || indptr == nullptr || indices == nullptr || last_page_len == nullptr ||
      out == nullptr || batch < 0 || num_pages <= 0 || num_kv_heads <= 0 || num_qo_heads % num_kv_heads != 0 ||
      num_splits < 1)
    return PL_ERR_INVALID_ARGUMENT;
  const int group = num_qo_heads / num_kv_heads;
  if (fold < 1 || (fused != nullptr && fold != 1)) return PL_ERR_INVALID_ARGUMENT;
  if (group * fold > 16 || (head_dim != 64 && head_dim != 128) || (page_size != 16 && page_size != 32))
    return PL_ERR_UNSUPPORTED;
  const int vrows = (batch + fold - 1) / fold;  // page-table rows
  if ((reinterpret_cast<uintptr_t>(kv_cache) & 15) != 0 || (reinterpret_cast<uintptr_t>(q) & 15) != 0 ||
      (q_stride_b % 8) != 0 || (q_stride_h % 8) != 0 ||
      (reinterpret_cast<uintptr_t>(out) & (out_is_f32 ? 15 : 7)) != 0 || (o_stride_b % 4) != 0 ||
      (o_stride_h % 4) != 0)
    return PL_ERR_INVALID_ARGUMENT;
  // counters per (page-table row, kv head), partial states per (query row, head);
  // a caller may reserve a fixed counter region so that shapes can alternate
  if (counter_bytes > 0 && counter_bytes < (int64_t)vrows * num_kv_heads * 4) return PL_ERR_WORKSPACE_TOO_SMALL;
  const int64_t c_bytes = counter_bytes > 0 ? counter_bytes : align256((int64_t)vrows * num_kv_heads * 4);
  const int64_t need = num_splits <= 1 ? c_bytes
                                       : c_bytes + align256((int64_t)batch * num_qo_heads * num_splits * head_dim * 4) +
                                             align256((int64_t)batch * num_qo_heads * num_splits * 4);
  if (num_splits > 1 && (workspace == nullptr || workspace_bytes < need)) return PL_ERR_WORKSPACE_TOO_SMALL;

  CUtensorMap map;
  int32_t st = pl_host::kv_tensor_map(kv_cache, num_pages, num_kv_heads, head_dim, page_size, &map);
  if (st != PL_OK) return st;

  pl::DecodeArgs a;
  a.q = static_cast<const pl::bf16*>(q);
  a.q_stride_b = q_stride_b;
  a.q_stride_h = q_stride_h;
  a.indptr = indptr;
  a.indices = indices;
  a.last_page_len = last_page_len;
  a.num_pages = num_pages;
  a.num_qo_heads = num_qo_heads;
  a.num_kv_heads = num_kv_heads;
  a.group = group;
  a.scale_log2 = sm_scale * pl::kLog2e;
  a.num_splits = num_splits;
  a.fold = fold;
  a.rows_real = batch;
  a.cluster = use_cluster_merge(head_dim, page_size, num_splits, (int64_t)vrows * num_kv_heads) ? 1 : 0;
  a.fused = fused != nullptr ? 1 : 0;
  a.qh = fused != nullptr ? *fused : pl::QkvHeadArgs{};
  a.slot_page = slot_page;
  a.slot_off = slot_off;
  a.cache_w = static_cast<pl::bf16*>(const_cast<void*>(kv_cache));
  a.q_out = static_cast<pl::bf16*>(q_out);
  a.out = out_is_f32 ? nullptr : static_cast<pl::bf16*>(out);
  a.out_f32 = out_is_f32 ? static_cast<float*>(out) : nullptr;
  a.o_stride_b = o_stride_b;
  a.o_stride_h = o_stride_h;
  a.out_lse = out_lse;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.counters = reinterpret_cast<int32_t*>(ws);
  a.partial_o = nullptr;
  a.partial_lse = nullptr;
  if (num_splits > 1) {
    const int64_t o_bytes = align256((int64_t)batch * num_qo_heads * num_splits * head_dim * 4);
    a.partial_o = reinterpret_cast<float*>(ws + c_bytes);
    a.partial_lse = reinterpret_cast<float*>(ws + c_bytes + o_bytes);
  }
  a.status = status_dev;
  a.prior_o = prior_o;
  a.prior_lse = prior_lse;

  if (head_dim == 128 && page_size == 16) return launch_decode<128, 16>(map, a, vrows, num_kv_heads, num_splits, stream);
  if (head_dim == 128 && page_size == 32) return launch_decode<128, 32>(map, a, vrows, num_kv_heads, num_splits, stream);
  if (head_dim == 64 && page_size == 16) return launch_decode<64, 16>(map, a, vrows, num_kv_heads, num_splits, stream);
  return launch_decode<64, 32>(map, a, vrows, num_kv_heads, num_splits, stream);
}
}  // namespace

extern "C" int32_t pl_paged_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* kv_cache,
                                   int64_t num_pages, const int32_t* indptr, const int32_t* indices,
                                   const int32_t* last_page_len, int32_t batch, int32_t num_qo_heads,
                                   int32_t num_kv_heads, int32_t head_dim, int32_t page_size, float sm_scale,
                                   int32_t num_splits, void* out, int64_t o_stride_b, int64_t o_stride_h,
                                   float* out_lse, void* workspace, int64_t workspace_bytes, int32_t* status_dev,
                                   void* stream) {
  return paged_decode_impl(q, q_stride_b, q_stride_h, kv_cache, num_pages, indptr, indices, last_page_len, batch,
                           num_qo_heads, num_kv_heads, head_dim, page_size, sm_scale, num_splits, out, false,
                           o_stride_b, o_stride_h, out_lse, workspace, workspace_bytes, status_dev, stream);
}

extern "C" int32_t pl_paged_decode_f32(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* kv_cache,
                                       int64_t num_pages, const int32_t* indptr, const int32_t* indices,
                                       const int32_t* last_page_len, int32_t batch, int32_t num_qo_heads,
                                       int32_t num_kv_heads, int32_t head_dim, int32_t page_size, float sm_scale,
                                       int32_t num_splits, float* out, int64_t o_stride_b, int64_t o_stride_h,
                                       float* out_lse, void* workspace, int64_t workspace_bytes, int32_t* status_dev,
                                       void* stream) {
  return paged_decode_impl(q, q_stride_b, q_stride_h, kv_cache, num_pages, indptr, indices, last_page_len, batch,
                           num_qo_heads, num_kv_heads, head_dim, page_size, sm_scale, num_splits, out, true,
                           o_stride_b, o_stride_h, out_lse, workspace, workspace_bytes, status_dev, stream);
}

extern "C" int32_t pl_paged_decode_shared(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                          const void* kv_cache, int64_t num_pages, const int32_t* indptr,
                                          const int32_t* indices, const int32_t* last_page_len, int32_t batch,
                                          int32_t fold, int32_t num_qo_heads, int32_t num_kv_heads,
                                          int32_t head_dim, int32_t page_size, float sm_scale, int32_t num_splits,
                                          void* out, int64_t o_stride_b, int64_t o_stride_h, float* out_lse,
                                          int32_t flags, void* workspace, int64_t workspace_bytes,
                                          int32_t* status_dev, void* stream) {
  return paged_decode_impl(q, q_stride_b, q_stride_h, kv_cache, num_pages, indptr, indices, last_page_len, batch,
                           num_qo_heads, num_kv_heads, head_dim, page_size, sm_scale, num_splits, out,
                           (flags & PL_DECODE_OUT_F32) != 0, o_stride_b, o_stride_h, out_lse, workspace,
                           workspace_bytes, status_dev, stream, nullptr, nullptr, nullptr, nullptr, fold);
}

extern "C" int32_t pl_paged_decode_merge_prior(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                               const void* kv_cache, int64_t num_pages, const int32_t* indptr,
                                               const int32_t* indices, const int32_t* last_page_len, int32_t batch,
                                               int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
                                               int32_t page_size, float sm_scale, int32_t num_splits, void* out,
                                               int64_t o_stride_b, int64_t o_stride_h, const float* prior_o,
                                               const float* prior_lse, void* workspace, int64_t workspace_bytes,
                                               int32_t* status_dev, void* stream) {
  if (prior_o == nullptr || prior_lse == nullptr) return PL_ERR_INVALID_ARGUMENT;
  return paged_decode_impl(q, q_stride_b, q_stride_h, kv_cache, num_pages, indptr, indices, last_page_len, batch,
                           num_qo_heads, num_kv_heads, head_dim, page_size, sm_scale, num_splits, out, false,
                           o_stride_b, o_stride_h, nullptr, workspace, workspace_bytes, status_dev, stream, nullptr,
                           nullptr, nullptr, nullptr, 1, 0, prior_o, prior_lse);
}

extern "C" int32_t pl_paged_decode_qkv(const void* qkv, int64_t qkv_stride, const float* lora_down,
                                       int64_t down_stride, const void* lora_b, int32_t lora_rank, float lora_scale,
                                       const int32_t* tok_adapter, const void* q_norm_w, const void* k_norm_w,
                                       float norm_eps, const int32_t* positions, float rope_theta,
                                       const float* rope_cos_sin, const int32_t* slot_page,
                                       const int32_t* slot_offset, void* q_out,
                                       void* kv_cache, int64_t num_pages, const int32_t* indptr,
                                       const int32_t* indices, const int32_t* last_page_len, int32_t batch,
                                       int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim,
                                       int32_t page_size, float sm_scale, int32_t num_splits, void* out,
                                       int64_t o_stride_b, int64_t o_stride_h, float* out_lse, int32_t flags,
                                       void* workspace, int64_t workspace_bytes, int32_t* status_dev, void* stream) {
  pl::QkvHeadArgs h;
  h.qkv = static_cast<const pl::bf16*>(qkv);
  h.qkv_stride = qkv_stride;
  h.down = lora_down;
  h.down_stride = down_stride;
  h.lora_b = static_cast<const pl::bf16*>(lora_b);
  h.rank = lora_rank;
  h.lora_scale = lora_scale;
  h.tok_adapter = tok_adapter;
  h.q_norm_w = static_cast<const pl::bf16*>(q_norm_w);
  h.k_norm_w = static_cast<const pl::bf16*>(k_norm_w);
  h.eps = norm_eps;
  h.positions = positions;
  h.theta = rope_theta;
  h.rope_cs = rope_cos_sin;
  if (rope_cos_sin != nullptr && ((reinterpret_cast<uintptr_t>(rope_cos_sin) & 15) || head_dim % 32))
    return PL_ERR_UNSUPPORTED;
  h.Hq = num_qo_heads;
  h.Hkv = num_kv_heads;
  return paged_decode_impl(nullptr, 0, 0, kv_cache, num_pages, indptr, indices, last_page_len, batch, num_qo_heads,
                           num_kv_heads, head_dim, page_size, sm_scale, num_splits, out,
                           (flags & PL_DECODE_OUT_F32) != 0, o_stride_b, o_stride_h, out_lse, workspace,
                           workspace_bytes, status_dev, stream, &h, slot_page, slot_offset, q_out);
}

extern "C" int32_t pl_decode_cluster_capacity(int32_t head_dim, int32_t page_size, int32_t num_splits) {
  if (num_splits < 2 || num_splits > kMaxClusterSplits) return 0;
  return cluster_capacity_for(head_dim, page_size, num_splits);
}

extern "C" int32_t pl_decode_set_cluster_merge(int32_t enable) {
  g_cluster_merge = enable != 0;
  return PL_OK;
}

extern "C" int32_t pl_merge_states_strided(const float* v_partial, int64_t v_row_stride, int64_t v_state_stride,
                                           const float* lse_partial, int64_t lse_row_stride,
                                           int64_t lse_state_stride, int32_t num_rows, int32_t num_states,
                                           int32_t head_dim, void* out, int64_t out_stride, float* out_lse,
                                           void* stream) {
  if (num_rows == 0) return PL_OK;
  if (v_partial == nullptr || lse_partial == nullptr || out == nullptr || num_rows < 0 || num_states < 1 ||
      head_dim <= 0)
    return PL_ERR_INVALID_ARGUMENT;
  return pl_host::launch_pdl(pl::merge_states_strided_kernel, dim3(num_rows), dim3(128), 0, stream, v_partial,
                             v_row_stride, v_state_stride, lse_partial, lse_row_stride, lse_state_stride,
                             (int)num_rows, (int)num_states, (int)head_dim, static_cast<pl::bf16*>(out), out_stride,
                             out_lse);
}

extern "C" int32_t pl_merge_states(const float* v_partial, const float* lse_partial, int32_t num_rows,
                                   int32_t num_states, int32_t head_dim, void* out, int64_t out_stride,
                                   float* out_lse, void* stream) {
  if (num_rows == 0) return PL_OK;
  if (v_partial == nullptr || lse_partial == nullptr || out == nullptr || num_rows < 0 || num_states < 1 ||
      head_dim <= 0)
    return PL_ERR_INVALID_ARGUMENT;
  return pl_host::launch_pdl(pl::merge_states_kernel, dim3(num_rows), dim3(128), 0, stream, v_partial, lse_partial,
                             (int)num_rows, (int)num_states, (int)head_dim, static_cast<pl::bf16*>(out), out_stride,
                             out_lse);
}

// ------------------------------------------------- fixed-scratch variant
// pl_paged_decode_fixed_scratch: the same kernel, with its split partials
// and arrival counters in a file-scope device array instead of a caller
// workspace, for callers that cannot allocate device memory.  One array per
// context (a __device__ variable exists once in every context that loads
// the library's module); its address is looked up, and the whole array
// cleared on the caller's stream, by the first call on each device and again
// whenever that device's current context is a different one (after a
// device reset the module is loaded anew and the array may move).  A fresh
// module's array is zero already; the clear is a defensive reset.  Its first
// kFixedCounterBytes hold the arrival counters whatever the shape, so that
// calls of different shapes may follow one another (a shape-sized counter
// region would let one call's partials land on another's counters).

static __device__ __align__(256) uint8_t g_decode_fixed_scratch[PL_FIXED_SCRATCH_BYTES];
constexpr int64_t kFixedCounterBytes = 64 * 1024;  // (row, kv head) pairs up to 16384

namespace {
constexpr int kScratchDevices = 64;
std::mutex g_fixed_scratch_mu;
void* g_fixed_scratch_ptr[kScratchDevices] = {};
void* g_fixed_scratch_ctx[kScratchDevices] = {};

using CtxGetCurrentFn = int (*)(void**);  // cuCtxGetCurrent (CUresult, CUcontext*)

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

int32_t fixed_scratch(void* stream, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return pl_host::record_cuda_error(e);
  if (dev < 0 || dev >= kScratchDevices) return PL_ERR_UNSUPPORTED;
  const CtxGetCurrentFn get_ctx = ctx_get_current_fn();
  if (get_ctx == nullptr) return PL_ERR_CUDA;
  void* ctx = nullptr;
  if (get_ctx(&ctx) != 0) return PL_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_fixed_scratch_mu);
  if (ctx != nullptr && ctx == g_fixed_scratch_ctx[dev] && g_fixed_scratch_ptr[dev] != nullptr) {
    *out = g_fixed_scratch_ptr[dev];
    return PL_OK;
  }
  // First call on this device, a host thread with no context bound yet, or
  // a new context: look the array up (this binds the device's primary
  // context when none is current) and clear it only if its context is new.
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_decode_fixed_scratch);
  if (e != cudaSuccess) return pl_host::record_cuda_error(e);
  if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 255)) return PL_ERR_CUDA;
  if (get_ctx(&ctx) != 0 || ctx == nullptr) return PL_ERR_CUDA;
  if (ctx != g_fixed_scratch_ctx[dev] || p != g_fixed_scratch_ptr[dev]) {
    // The counters at the front must start at zero; every completed call leaves them so.
    e = cudaMemsetAsync(p, 0, PL_FIXED_SCRATCH_BYTES, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return pl_host::record_cuda_error(e);
    g_fixed_scratch_ptr[dev] = p;
    g_fixed_scratch_ctx[dev] = ctx;
  }
  *out = p;
  return PL_OK;
}
}  // namespace

extern "C" int32_t pl_fixed_scratch_clear(void* stream) {
  void* scratch = nullptr;
  int32_t st = fixed_scratch(stream, &scratch);
  if (st != PL_OK) return st;
  const cudaError_t e = cudaMemsetAsync(scratch, 0, kFixedCounterBytes, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PL_OK : pl_host::record_cuda_error(e);
}

extern "C" int32_t pl_paged_decode_fixed_scratch(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                                 const void* kv_cache, int64_t num_pages, const int32_t* indptr,
                                                 const int32_t* indices, const int32_t* last_page_len,
                                                 int32_t batch, int32_t num_qo_heads, int32_t num_kv_heads,
                                                 int32_t head_dim, int32_t page_size, float sm_scale,
                                                 int32_t num_splits, void* out, int64_t o_stride_b,
                                                 int64_t o_stride_h, float* out_lse, int32_t* status_dev,
                                                 void* stream) {
  if (batch == 0) return PL_OK;
  if (batch < 0 || num_kv_heads <= 0 || num_qo_heads <= 0 || head_dim <= 0 || num_splits < 1)
    return PL_ERR_INVALID_ARGUMENT;
  const int64_t partial_bytes =
      num_splits <= 1 ? 0
                      : align256((int64_t)batch * num_qo_heads * num_splits * head_dim * 4) +
                            align256((int64_t)batch * num_qo_heads * num_splits * 4);
  if ((int64_t)batch * num_kv_heads * 4 > kFixedCounterBytes ||
      kFixedCounterBytes + partial_bytes > PL_FIXED_SCRATCH_BYTES)
    return PL_ERR_WORKSPACE_TOO_SMALL;
  void* scratch = nullptr;
  int32_t st = fixed_scratch(stream, &scratch);
  if (st != PL_OK) return st;
  return paged_decode_impl(q, q_stride_b, q_stride_h, kv_cache, num_pages, indptr, indices, last_page_len, batch,
                           num_qo_heads, num_kv_heads, head_dim, page_size, sm_scale, num_splits, out, false,
                           o_stride_b, o_stride_h, out_lse, scratch, PL_FIXED_SCRATCH_BYTES, status_dev, stream,
                           nullptr, nullptr, nullptr, nullptr, 1, kFixedCounterBytes);
}
