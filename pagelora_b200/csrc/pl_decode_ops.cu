// Page-table construction and the small per-token kernels of one decode
// step: q/k head RMSNorm + RoPE + paged KV append, the plain KV append,
// embedding gather and first-index argmax.
#include "pl_qkv_head.cuh"

namespace pl {

constexpr int kPtThreads = 1024;
constexpr int kPtMaxRows = 4096;

// Warp-uniform scan state of one row of spans.
struct RowScan {
  bool have_prev;
  int32_t prev_blk, prev_end;
  bool open;
  int32_t open_start;
  long long open_sum;
  int32_t n_groups;
};

// Pass 1 of the page-table build for one row (one warp): coalesce adjacent
// slices of one page (flashinfer_page_table.py:184-197), validate every
// coalesced span in order (:210-220) and count them.  Returns the status
// kind of the first failing coalesced span (0 if none) and the last length.
__device__ int32_t pt_scan_row(const int32_t* blk, const int32_t* st, const int32_t* ln, int32_t s0, int32_t s1,
                               int32_t PS, int32_t* n_groups_out, int32_t* last_len_out) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  RowScan rs = {false, 0, 0, false, 0, 0, 0};
  int32_t err = 0;
  for (int32_t c = s0; c < s1; c += 32) {
    const int32_t i = c + lane;
    const bool in = i < s1;
    const int32_t b = in ? blk[i] : 0;
    const int32_t s = in ? st[i] : 0;
    const int32_t l = in ? ln[i] : 0;
    const bool ne = in && l > 0;  // empty slices are skipped by the coalescer
    const uint32_t M = __ballot_sync(0xffffffffu, ne);
    const uint32_t below = M & lt;
    const int jp = below ? 31 - __clz(below) : lane;
    const int32_t pb_l = __shfl_sync(0xffffffffu, b, jp);
    const int32_t pe_l = __shfl_sync(0xffffffffu, s + l, jp);
    const bool hp = below ? true : rs.have_prev;
    const int32_t pb = below ? pb_l : rs.prev_blk;
    const int32_t pe = below ? pe_l : rs.prev_end;
    const bool cont = ne && hp && b == pb && s == pe;
    const bool head = ne && !cont;
    const uint32_t H = __ballot_sync(0xffffffffu, head);
    long long P = ne ? (long long)l : 0ll;
    const long long val = P;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, P, o);
      if (lane >= o) P += y;
    }
    const long long Pex = P - val;
    const uint32_t hbelow = H & lt;
    const int hl = hbelow ? 31 - __clz(hbelow) : lane;
    const int32_t hp_start = __shfl_sync(0xffffffffu, s, hl);
    const long long hp_pex = __shfl_sync(0xffffffffu, Pex, hl);
    int32_t kind = 0;
    if (head) {
      bool closes = false;
      int32_t cstart = 0;
      long long clen = 0;
      if (hbelow) {
        closes = true;
        cstart = hp_start;
        clen = Pex - hp_pex;
      } else if (rs.open) {
        closes = true;
        cstart = rs.open_start;
        clen = rs.open_sum + Pex;
      }
      if (closes) {  // a head follows, so the closed span is not the row's last
        if (cstart != 0)
          kind = PL_ERR_SPAN_START;
        else if (clen <= 0 || clen > PS)
          kind = PL_ERR_SPAN_LENGTH;
        else if (clen != PS)
          kind = PL_ERR_SPAN_NOT_FULL;
      }
    }
    const uint32_t E = __ballot_sync(0xffffffffu, kind != 0);
    if (E) {
      err = __shfl_sync(0xffffffffu, kind, __ffs(E) - 1);
      break;
    }
    const long long Ptot = __shfl_sync(0xffffffffu, P, 31);
    if (H) {
      const int hh = 31 - __clz(H);
      rs.open = true;
      rs.open_start = __shfl_sync(0xffffffffu, s, hh);
      rs.open_sum = Ptot - __shfl_sync(0xffffffffu, Pex, hh);
    } else if (rs.open) {
      rs.open_sum += Ptot;
    }
    rs.n_groups += __popc(H);
    if (M) {
      const int ln_ = 31 - __clz(M);
      rs.have_prev = true;
      rs.prev_blk = __shfl_sync(0xffffffffu, b, ln_);
      rs.prev_end = __shfl_sync(0xffffffffu, s + l, ln_);
    }
  }
  if (err == 0 && rs.open) {  // the row's last coalesced span may be partial
    if (rs.open_start != 0)
      err = PL_ERR_SPAN_START;
    else if (rs.open_sum <= 0 || rs.open_sum > PS)
      err = PL_ERR_SPAN_LENGTH;
  }
  *n_groups_out = rs.n_groups;
  *last_len_out = rs.open ? (int32_t)rs.open_sum : 0;
  return err;
}

// Pass 2: write the page id of every coalesced span of one row.
__device__ void pt_write_row(const int32_t* blk, const int32_t* st, const int32_t* ln, int32_t s0, int32_t s1,
                             int32_t* out) {
  const int lane = threadIdx.x & 31;
  const uint32_t lt = (1u << lane) - 1u;
  bool have_prev = false;
  int32_t prev_blk = 0, prev_end = 0, n_groups = 0;
  for (int32_t c = s0; c < s1; c += 32) {
    const int32_t i = c + lane;
    const bool in = i < s1;
    const int32_t b = in ? blk[i] : 0;
    const int32_t s = in ? st[i] : 0;
    const int32_t l = in ? ln[i] : 0;
    const bool ne = in && l > 0;
    const uint32_t M = __ballot_sync(0xffffffffu, ne);
    const uint32_t below = M & lt;
    const int jp = below ? 31 - __clz(below) : lane;
    const int32_t pb_l = __shfl_sync(0xffffffffu, b, jp);
    const int32_t pe_l = __shfl_sync(0xffffffffu, s + l, jp);
    const bool hp = below ? true : have_prev;
    const int32_t pb = below ? pb_l : prev_blk;
    const int32_t pe = below ? pe_l : prev_end;
    const bool head = ne && !(hp && b == pb && s == pe);
    const uint32_t H = __ballot_sync(0xffffffffu, head);
    if (head) out[n_groups + __popc(H & lt)] = b;
    n_groups += __popc(H);
    if (M) {
      const int ln_ = 31 - __clz(M);
      have_prev = true;
      prev_blk = __shfl_sync(0xffffffffu, b, ln_);
      prev_end = __shfl_sync(0xffffffffu, s + l, ln_);
    }
  }
}

// Block-wide exclusive scan of vals[0..n) (n <= kPtMaxRows) in place; returns the total.
__device__ int32_t block_exclusive_scan(int32_t* vals, int n, int32_t* tmp32) {
  constexpr int kPer = kPtMaxRows / kPtThreads;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int32_t loc[kPer];
  int32_t sum = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int r = tid * kPer + i;
    loc[i] = r < n ? vals[r] : 0;
    sum += loc[i];
  }
  int32_t inc = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) tmp32[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int32_t w = lane < (kPtThreads / 32) ? tmp32[lane] : 0;
    int32_t wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    tmp32[lane] = wi - w;  // exclusive warp offsets
    if (lane == 31) tmp32[32] = wi;
  }
  __syncthreads();
  int32_t run = tmp32[warp] + inc - sum;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int r = tid * kPer + i;
    if (r < n) vals[r] = run;
    run += loc[i];
  }
  const int32_t total = tmp32[32];
  __syncthreads();
  return total;
}

__global__ void __launch_bounds__(kPtThreads) page_table_build_kernel(
    const int32_t* __restrict__ blk, const int32_t* __restrict__ st, const int32_t* __restrict__ ln,
    const int32_t* __restrict__ row_indptr, int num_rows, int PS, int32_t* __restrict__ out_indptr,
    int32_t* __restrict__ out_indices, int32_t* __restrict__ out_last, int32_t* status, int32_t* err_row) {
  extern __shared__ int32_t pt_sm[];
  int32_t* counts = pt_sm;
  int32_t* lastl = pt_sm + num_rows;
  int32_t* errk = pt_sm + 2 * num_rows;
  __shared__ int32_t tmp32[33];
  __shared__ int32_t first_bad;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kWarps = kPtThreads / 32;
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x == 0) first_bad = num_rows;
  for (int r = warp; r < num_rows; r += kWarps) {
    int32_t ng = 0, ll = 0;
    const int32_t e = pt_scan_row(blk, st, ln, row_indptr[r], row_indptr[r + 1], PS, &ng, &ll);
    if (lane == 0) {
      counts[r] = ng;
      lastl[r] = ll;
      errk[r] = e;
    }
  }
  __syncthreads();
  for (int r = threadIdx.x; r < num_rows; r += kPtThreads)
    if (errk[r] != 0) atomicMin(&first_bad, r);
  __syncthreads();
  if (first_bad < num_rows) {
    if (threadIdx.x == 0) {
      if (status != nullptr) atomicCAS(status, 0, errk[first_bad]);
      if (err_row != nullptr) *err_row = first_bad;
    }
    return;
  }
  const int32_t total = block_exclusive_scan(counts, num_rows, tmp32);
  for (int r = threadIdx.x; r < num_rows; r += kPtThreads) {
    out_indptr[r] = counts[r];
    out_last[r] = lastl[r];
  }
  if (threadIdx.x == 0) out_indptr[num_rows] = total;
  for (int r = warp; r < num_rows; r += kWarps)
    pt_write_row(blk, st, ln, row_indptr[r], row_indptr[r + 1], out_indices + counts[r]);
}

// One decode token per row: extend the row by one slot (appending
// new_page_ids[r] when its last page is full or the row is empty), record
// the append slot, then rebuild the CSR page table from the per-row pages.
__global__ void __launch_bounds__(kPtThreads) page_table_advance_kernel(
    int32_t* __restrict__ row_num_pages, int32_t* __restrict__ last_page_len, int32_t* __restrict__ row_pages,
    const int32_t* __restrict__ new_page_ids, int num_rows, int cap, int PS, int32_t* __restrict__ out_indptr,
    int32_t* __restrict__ out_indices, int32_t* __restrict__ slot_page, int32_t* __restrict__ slot_off,
    int32_t* __restrict__ positions, int32_t* status) {
  extern __shared__ int32_t pt_sm[];
  int32_t* counts = pt_sm;
  __shared__ int32_t tmp32[33];
  pdl_launch_dependents();
  pdl_wait();
  for (int r = threadIdx.x; r < num_rows; r += kPtThreads) {
    int32_t n = row_num_pages[r];
    int32_t last = last_page_len[r];
    if (n == 0 || last >= PS) {
      if (n >= cap) {
        set_status(status, PL_ERR_INVALID_ARGUMENT);
        counts[r] = n;
        slot_page[r] = -1;
        slot_off[r] = 0;
        continue;
      }
      row_pages[(int64_t)r * cap + n] = new_page_ids[r];
      ++n;
      last = 1;
    } else {
      ++last;
    }
    row_num_pages[r] = n;
    last_page_len[r] = last;
    slot_page[r] = row_pages[(int64_t)r * cap + n - 1];
    slot_off[r] = last - 1;
    if (positions != nullptr) positions[r] = (n - 1) * PS + last - 1;
    counts[r] = n;
  }
  __syncthreads();
  const int32_t total = block_exclusive_scan(counts, num_rows, tmp32);
  for (int r = threadIdx.x; r < num_rows; r += kPtThreads) out_indptr[r] = counts[r];
  if (threadIdx.x == 0) out_indptr[num_rows] = total;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < num_rows; r += kPtThreads / 32) {
    const int32_t off = counts[r];
    const int32_t n = (r + 1 < num_rows ? counts[r + 1] : total) - off;
    for (int i = lane; i < n; i += 32) out_indices[off + i] = row_pages[(int64_t)r * cap + i];
  }
}

// ---------------------------------------------------------------- KV append
__global__ void kv_append_kernel(const bf16* __restrict__ k, int64_t k_stride, const bf16* __restrict__ v,
                                 int64_t v_stride, bf16* __restrict__ cache, int64_t num_pages,
                                 const int32_t* __restrict__ page_id, const int32_t* __restrict__ page_off, int T,
                                 int Hkv, int D, int PS, int32_t* status) {
  pdl_launch_dependents();
  pdl_wait();
  const int per_tok = Hkv * D / 8;
  const int64_t total = (int64_t)T * per_tok;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < total; c += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(c / per_tok);
    const int rem = (int)(c % per_tok);
    const int32_t pid = page_id[t], off = page_off[t];
    if (pid < 0 || pid >= num_pages || off < 0 || off >= PS) {
      set_status(status, PL_ERR_PAGE_OUT_OF_RANGE);
      continue;
    }
    const int64_t kbase = (((int64_t)pid * 2 + 0) * PS + off) * Hkv * D;
    const int64_t vbase = (((int64_t)pid * 2 + 1) * PS + off) * Hkv * D;
    const int e = rem * 8;  // element within [Hkv*D]
    *reinterpret_cast<uint4*>(cache + kbase + e) = *reinterpret_cast<const uint4*>(k + t * k_stride + e);
    *reinterpret_cast<uint4*>(cache + vbase + e) = *reinterpret_cast<const uint4*>(v + t * v_stride + e);
  }
}

// ------------------------------------------- q/k norm + RoPE + KV append
// One warp per (token, head) over the packed [q | k | v] projection row.
template <int D>
__global__ void __launch_bounds__(128) qkv_rope_append_kernel(const QkvHeadArgs a, bf16* __restrict__ q_out,
                                                              bf16* __restrict__ cache, int64_t num_pages,
                                                              const int32_t* __restrict__ page_id,
                                                              const int32_t* __restrict__ page_off, int T, int PS,
                                                              int32_t* status) {
  constexpr int E = D / 32;
  if (threadIdx.x == 0) PL_TRACE_POINT(0);
  pdl_launch_dependents();
  const int heads = a.Hq + 2 * a.Hkv;
  const int gw = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (gw < T * heads) qkv_head_prefetch<D>(a, gw % heads, lane);
  pdl_wait();
  if (threadIdx.x == 0) PL_TRACE_POINT(1);
  if (gw >= T * heads) return;
  const int t = gw / heads, hh = gw % heads;
  const int d0 = lane * E;
  float v[E];
  qkv_head_transform<D>(a, t, hh, lane, v);
  if (lane == 0) PL_TRACE_MAX(2);
  if (hh < a.Hq) {
    bf16* dst = q_out + ((int64_t)t * a.Hq + hh) * D + d0;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = f2bf(v[e]);
  } else {
    const int32_t pid = page_id[t], off = page_off[t];
    if (pid < 0 || pid >= num_pages || off < 0 || off >= PS) {
      if (lane == 0) set_status(status, PL_ERR_PAGE_OUT_OF_RANGE);
      return;
    }
    const int kv = hh < a.Hq + a.Hkv ? 0 : 1;
    const int h = hh - a.Hq - kv * a.Hkv;
    bf16* dst = cache + ((((int64_t)pid * 2 + kv) * PS + off) * a.Hkv + h) * D + d0;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = f2bf(v[e]);
  }
}

// ----------------------------------------------------------------- embed
__global__ void embed_kernel(const int64_t* __restrict__ ids, const bf16* __restrict__ table, int64_t vocab, int dim,
                             bf16* __restrict__ out, int32_t* status) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const int64_t id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) set_status(status, PL_ERR_INVALID_ARGUMENT);
    return;
  }
  for (int c = threadIdx.x; c < dim / 8; c += blockDim.x)
    reinterpret_cast<uint4*>(out + (int64_t)t * dim)[c] = reinterpret_cast<const uint4*>(table + id * dim)[c];
}

// ---------------------------------------------------------------- argmax
// (value, index) ordering of torch.argmax: larger value wins, NaN beats any
// number, ties go to the smaller index.
__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn || bn) return vn && (!bn || i < bi);
  return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void am_block_reduce(float& best, int& bi, float* sv, int* si) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (am_better(ov, oi, best, bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x / 32;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (am_better(ov, oi, best, bi)) {
        best = ov;
        bi = oi;
      }
    }
  }
}

// grid (chunks, tokens): each CTA scans one vocab chunk and leaves a
// candidate; the last CTA of a token (arrival ticket) reduces the
// candidates in chunk order and resets the ticket.
__global__ void __launch_bounds__(256) argmax_kernel(const bf16* __restrict__ logits, int64_t stride, int vocab,
                                                     int chunk, int64_t* __restrict__ out, float* cand_v,
                                                     int* cand_i, int* tickets) {
  pdl_launch_dependents();
  pdl_wait();
  const int c = blockIdx.x, t = blockIdx.y, nc = gridDim.x;
  const bf16* row = logits + (int64_t)t * stride;
  const int i0 = c * chunk, i1 = min(vocab, i0 + chunk);
  float best = -INFINITY;
  int bi = 0x7fffffff;
  const bool vec = ((reinterpret_cast<uintptr_t>(row) | (uintptr_t)(i0 * 2)) & 15) == 0;
  if (vec) {
    for (int i = i0 + threadIdx.x * 8; i < i1; i += blockDim.x * 8) {
      if (i + 8 <= i1) {
        const uint4 u = *reinterpret_cast<const uint4*>(row + i);
        const uint32_t* w = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(w[q]);
          if (am_better(f.x, i + 2 * q, best, bi)) { best = f.x; bi = i + 2 * q; }
          if (am_better(f.y, i + 2 * q + 1, best, bi)) { best = f.y; bi = i + 2 * q + 1; }
        }
      } else {
        for (int j = i; j < i1; ++j) {
          const float v = bf2f(row[j]);
          if (am_better(v, j, best, bi)) { best = v; bi = j; }
        }
      }
    }
  } else {
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
      const float v = bf2f(row[i]);
      if (am_better(v, i, best, bi)) { best = v; bi = i; }
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ int is_last;
  am_block_reduce(best, bi, sv, si);
  if (threadIdx.x == 0) {
    cand_v[t * nc + c] = best;
    cand_i[t * nc + c] = bi;
    __threadfence();
    is_last = atomicAdd(&tickets[t], 1) == nc - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  best = -INFINITY;
  bi = 0x7fffffff;
  for (int k = threadIdx.x; k < nc; k += blockDim.x) {
    const float v = __ldcg(cand_v + t * nc + k);
    const int i = __ldcg(cand_i + t * nc + k);
    if (am_better(v, i, best, bi)) { best = v; bi = i; }
  }
  __syncthreads();
  am_block_reduce(best, bi, sv, si);
  if (threadIdx.x == 0) {
    out[t] = bi == 0x7fffffff ? 0 : bi;
    tickets[t] = 0;
  }
}

// Hugging Face RMSNorm rounding (Qwen3 q/k head norm, LlamaRMSNorm):
// y = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))), one warp per row of K
// elements (K % 8 == 0), 8 rows per CTA.
__global__ void __launch_bounds__(256) rmsnorm_hf_kernel(const bf16* __restrict__ x, int64_t x_stride, int rows,
                                                         int K, const bf16* __restrict__ w, float eps,
                                                         bf16* __restrict__ y, int64_t y_stride) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bf16* xr = x + (int64_t)row * x_stride;
  float ss = 0.f;
  for (int k = lane * 8; k < K; k += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
    const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = unpack_bf16x2(u[q]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)K + eps);
  for (int k = lane * 8; k < K; k += 256) {
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
      const float2 n = unpack_bf16x2(pack_bf16x2(f.x * r, f.y * r));
      uo[q] = pack_bf16x2(gw.x * n.x, gw.y * n.y);
    }
    *reinterpret_cast<uint4*>(y + (int64_t)row * y_stride + k) = out;
  }
}

// (cos, sin) of every RoPE angle of every row's position: [rows][D/2][2]
// fp32.  Positions are the same for all layers of a decode step, so the
// step's launches read this table instead of evaluating powf / sincosf per
// layer (the same rope_angle_cs, hence the same values).
__global__ void rope_cos_sin_kernel(const int32_t* __restrict__ positions, int half, int D, float theta,
                                    float* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int row = blockIdx.x;
  const float pos = (float)positions[row];
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float cs, sn;
    rope_angle_cs(pos, i, D, theta, cs, sn);
    *reinterpret_cast<float2*>(out + ((int64_t)row * half + i) * 2) = make_float2(cs, sn);
  }
}

}  // namespace pl

// =================================================================== host
PL_TRACE_READER(pl_trace_read_ops)
extern "C" int32_t pl_page_table_build(const int32_t* span_block_id, const int32_t* span_start,
                                       const int32_t* span_length, const int32_t* row_indptr, int32_t num_rows,
                                       int32_t page_size, int32_t* out_indptr, int32_t* out_indices,
                                       int32_t* out_last_page_len, int32_t* status_dev, int32_t* err_row_dev,
                                       void* stream) {
  if (num_rows < 0 || page_size <= 0 || row_indptr == nullptr || out_indptr == nullptr || status_dev == nullptr)
    return PL_ERR_INVALID_ARGUMENT;
  if (num_rows > pl::kPtMaxRows) return PL_ERR_UNSUPPORTED;
  if (num_rows > 0 && (span_block_id == nullptr || span_start == nullptr || span_length == nullptr ||
                       out_indices == nullptr || out_last_page_len == nullptr))
    return PL_ERR_INVALID_ARGUMENT;
  const int smem = 3 * (num_rows > 0 ? num_rows : 1) * 4;
  int32_t st = pl_host::ensure_smem_attr(reinterpret_cast<const void*>(pl::page_table_build_kernel), smem);
  if (st != PL_OK) return st;
  return pl_host::launch_pdl(pl::page_table_build_kernel, dim3(1), dim3(pl::kPtThreads), smem, stream,
                             span_block_id, span_start, span_length, row_indptr, (int)num_rows, (int)page_size,
                             out_indptr, out_indices, out_last_page_len, status_dev, err_row_dev);
}

extern "C" int32_t pl_page_table_advance(int32_t* row_num_pages, int32_t* last_page_len, int32_t* row_pages,
                                         const int32_t* new_page_ids, int32_t num_rows, int32_t row_capacity,
                                         int32_t page_size, int32_t* out_indptr, int32_t* out_indices,
                                         int32_t* slot_page_id, int32_t* slot_offset, int32_t* positions_out,
                                         int32_t* status_dev, void* stream) {
  if (num_rows == 0) return PL_OK;
  if (row_num_pages == nullptr || last_page_len == nullptr || row_pages == nullptr || new_page_ids == nullptr ||
      out_indptr == nullptr || out_indices == nullptr || slot_page_id == nullptr || slot_offset == nullptr ||
      num_rows < 0 || row_capacity <= 0 || page_size <= 0)
    return PL_ERR_INVALID_ARGUMENT;
  if (num_rows > pl::kPtMaxRows) return PL_ERR_UNSUPPORTED;
  return pl_host::launch_pdl(pl::page_table_advance_kernel, dim3(1), dim3(pl::kPtThreads), (size_t)num_rows * 4,
                             stream, row_num_pages, last_page_len, row_pages, new_page_ids, (int)num_rows,
                             (int)row_capacity, (int)page_size, out_indptr, out_indices, slot_page_id, slot_offset,
                             positions_out, status_dev);
}

extern "C" int32_t pl_kv_append(const void* k, int64_t k_stride, const void* v, int64_t v_stride, void* kv_cache,
                                int64_t num_pages, const int32_t* page_id, const int32_t* page_offset,
                                int32_t num_tokens, int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
                                int32_t* status_dev, void* stream) {
  if (num_tokens == 0) return PL_OK;
  if (k == nullptr || v == nullptr || kv_cache == nullptr || page_id == nullptr || page_offset == nullptr ||
      num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || page_size <= 0)
    return PL_ERR_INVALID_ARGUMENT;
  if ((num_kv_heads * head_dim) % 8 || (k_stride % 8) || (v_stride % 8) || (reinterpret_cast<uintptr_t>(k) & 15) ||
      (reinterpret_cast<uintptr_t>(v) & 15) || (reinterpret_cast<uintptr_t>(kv_cache) & 15))
    return PL_ERR_UNSUPPORTED;
  const int64_t chunks = (int64_t)num_tokens * num_kv_heads * head_dim / 8;
  const int blocks = (int)((chunks + 255) / 256 < 4096 ? (chunks + 255) / 256 : 4096);
  return pl_host::launch_pdl(pl::kv_append_kernel, dim3(blocks), dim3(256), 0, stream,
                             static_cast<const pl::bf16*>(k), k_stride, static_cast<const pl::bf16*>(v), v_stride,
                             static_cast<pl::bf16*>(kv_cache), num_pages, page_id, page_offset, (int)num_tokens,
                             (int)num_kv_heads, (int)head_dim, (int)page_size, status_dev);
}

extern "C" int32_t pl_qkv_rope_append(const void* qkv, int64_t qkv_stride, const float* lora_down,
                                      int64_t down_stride, const void* lora_b, int32_t lora_rank,
                                      float lora_scale,
                                      const int32_t* tok_adapter, const void* q_norm_w, const void* k_norm_w,
                                      float norm_eps, const int32_t* positions, float rope_theta, void* q_out,
                                      void* kv_cache, int64_t num_pages, const int32_t* page_id,
                                      const int32_t* page_offset, int32_t num_tokens, int32_t num_qo_heads,
                                      int32_t num_kv_heads, int32_t head_dim, int32_t page_size, int32_t* status_dev,
                                      void* stream) {
  if (num_tokens == 0) return PL_OK;
  if (qkv == nullptr || positions == nullptr || q_out == nullptr || kv_cache == nullptr || page_id == nullptr ||
      page_offset == nullptr || num_tokens < 0 || num_qo_heads <= 0 || num_kv_heads <= 0 || page_size <= 0)
    return PL_ERR_INVALID_ARGUMENT;
  if (lora_down != nullptr && lora_b != nullptr && lora_rank <= 0) return PL_ERR_INVALID_ARGUMENT;
  pl::QkvHeadArgs a;
  a.qkv = static_cast<const pl::bf16*>(qkv);
  a.qkv_stride = qkv_stride;
  a.down = lora_down;
  a.down_stride = down_stride;
  a.lora_b = static_cast<const pl::bf16*>(lora_b);
  a.rank = lora_rank;
  a.lora_scale = lora_scale;
  a.tok_adapter = tok_adapter;
  a.q_norm_w = static_cast<const pl::bf16*>(q_norm_w);
  a.k_norm_w = static_cast<const pl::bf16*>(k_norm_w);
  a.eps = norm_eps;
  a.positions = positions;
  a.theta = rope_theta;
  a.rope_cs = nullptr;
  a.Hq = num_qo_heads;
  a.Hkv = num_kv_heads;
  const int warps = num_tokens * (num_qo_heads + 2 * num_kv_heads);
  const int blocks = (warps + 3) / 4;
  if (head_dim == 128)
    return pl_host::launch_pdl(pl::qkv_rope_append_kernel<128>, dim3(blocks), dim3(128), 0, stream, a,
                               static_cast<pl::bf16*>(q_out), static_cast<pl::bf16*>(kv_cache), num_pages, page_id,
                               page_offset, (int)num_tokens, (int)page_size, status_dev);
  if (head_dim == 64)
    return pl_host::launch_pdl(pl::qkv_rope_append_kernel<64>, dim3(blocks), dim3(128), 0, stream, a,
                               static_cast<pl::bf16*>(q_out), static_cast<pl::bf16*>(kv_cache), num_pages, page_id,
                               page_offset, (int)num_tokens, (int)page_size, status_dev);
  return PL_ERR_UNSUPPORTED;
}

extern "C" int32_t pl_embed(const int64_t* token_ids, const void* table, int64_t vocab, int32_t dim,
                            int32_t num_tokens, void* out, int32_t* status_dev, void* stream) {
  if (num_tokens == 0) return PL_OK;
  if (token_ids == nullptr || table == nullptr || out == nullptr || num_tokens < 0 || dim <= 0 || vocab <= 0)
    return PL_ERR_INVALID_ARGUMENT;
  if (dim % 8 || (reinterpret_cast<uintptr_t>(table) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return PL_ERR_UNSUPPORTED;
  return pl_host::launch_pdl(pl::embed_kernel, dim3(num_tokens), dim3(256), 0, stream, token_ids,
                             static_cast<const pl::bf16*>(table), vocab, (int)dim, static_cast<pl::bf16*>(out),
                             status_dev);
}

extern "C" int32_t pl_argmax(const void* logits, int64_t stride, int32_t vocab, int32_t num_tokens,
                             int64_t* out_ids, void* workspace, int64_t workspace_bytes, void* stream) {
  if (num_tokens == 0) return PL_OK;
  if (logits == nullptr || out_ids == nullptr || num_tokens < 0 || vocab <= 0 || num_tokens > 65535)
    return PL_ERR_INVALID_ARGUMENT;
  int sms = pl_host::sm_count();
  if (sms <= 0) sms = 148;
  int chunks = (int)((vocab + 2047) / 2048);
  if (chunks > sms) chunks = sms;
  if (chunks < 1) chunks = 1;
  const int chunk = (int)(((vocab + chunks - 1) / chunks + 7) / 8 * 8);
  chunks = (vocab + chunk - 1) / chunk;
  const int64_t need = (int64_t)num_tokens * 4 + (int64_t)num_tokens * chunks * 8;
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return PL_ERR_WORKSPACE_TOO_SMALL;
  int* tickets = static_cast<int*>(workspace);
  float* cand_v = reinterpret_cast<float*>(tickets + num_tokens);
  int* cand_i = reinterpret_cast<int*>(cand_v + (int64_t)num_tokens * chunks);
  return pl_host::launch_pdl(pl::argmax_kernel, dim3(chunks, num_tokens), dim3(256), 0, stream,
                             static_cast<const pl::bf16*>(logits), stride, (int)vocab, chunk, out_ids, cand_v, cand_i,
                             tickets);
}

extern "C" int32_t pl_rmsnorm_hf(const void* x, int64_t x_stride, int32_t num_rows, int32_t k_in, const void* w,
                                 float eps, void* y, int64_t y_stride, void* stream) {
  if (num_rows == 0) return PL_OK;
  if (x == nullptr || w == nullptr || y == nullptr || num_rows < 0 || k_in <= 0) return PL_ERR_INVALID_ARGUMENT;
  if (k_in % 8 || x_stride % 8 || y_stride % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return PL_ERR_UNSUPPORTED;
  return pl_host::launch_pdl(pl::rmsnorm_hf_kernel, dim3((num_rows + 7) / 8), dim3(256), 0, stream,
                             static_cast<const pl::bf16*>(x), x_stride, (int)num_rows, (int)k_in,
                             static_cast<const pl::bf16*>(w), eps, static_cast<pl::bf16*>(y), y_stride);
}

extern "C" int32_t pl_rope_cos_sin(const int32_t* positions, int32_t rows, int32_t head_dim, float rope_theta,
                                   float* cos_sin, void* stream) {
  if (rows == 0) return PL_OK;
  if (positions == nullptr || cos_sin == nullptr || rows < 0 || head_dim <= 0 || head_dim % 32 != 0)
    return PL_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(cos_sin) & 15) return PL_ERR_UNSUPPORTED;
  const int half = head_dim / 2;
  return pl_host::launch_pdl(pl::rope_cos_sin_kernel, dim3(rows), dim3(half < 1024 ? half : 1024), 0, stream,
                             positions, half, (int)head_dim, rope_theta, cos_sin);
}
