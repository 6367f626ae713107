// Split-KV exchange over NVLink peer memory for sm_100a.
//
// In split-KV decode every GPU holds a contiguous page range of each row's
// context and computes a partial attention state (O fp32, LSE) over it; the
// states of all GPUs are merged by log-sum-exp.  pl_splitkv_exchange_merge
// replaces the per-layer collective (an NCCL all-gather of the packed
// partials followed by a merge launch) with one kernel:
//
//   1. CTA c stores its slice of this GPU's partial (rows [c*rpc, (c+1)*rpc)
//      of O and LSE) straight into slot `rank` of every GPU's gather buffer
//      (plain st.global through CUDA IPC mappings of the peers' buffers; no
//      multicast, no library kernel touches peer memory);
//   2. threads 0..world-1 publish the CTA's epoch to flag [rank][c] of every
//      GPU with a release store at system scope, then each waits (acquire,
//      bounded) until peer p's flag [p][c] here has reached the same epoch;
//   3. the CTA merges its rows from the local gather buffer, in GPU order,
//      with the arithmetic of merge_states_strided_kernel, so the result is
//      bit-identical to the all-gather path and the same on every GPU.
//
// The gather buffer has two halves chosen by the epoch's parity: a peer can
// only write the half of exchange e + 2 after this GPU has published epoch
// e + 1, which it does after its merge of exchange e has finished, so no
// store can land in a half that is still being read.  Epochs are per CTA,
// kept on the device and advanced by the kernel, so the launch can be
// replayed from a CUDA graph; flags only grow and never need a reset.
#include <cstring>

#include "pl_common.cuh"

namespace pl {

constexpr int kExThreads = 128;

struct ExchangeArgs {
  const float* part;            // this GPU's packed partial: O [rows_h][D], then LSE [rows_h] (natural log)
  float* const* peer_gather;    // [world] gather buffer of every GPU (own one included): [2][world][n]
  int32_t* const* peer_flags;   // [world] flag array of every GPU: [world][ctas]
  const int32_t* flags_local;   // this GPU's flag array
  int32_t* epochs;              // [ctas] this GPU's per-CTA epoch
  bf16* out;                    // [rows_h][D] merged attention output
  int32_t* status;
  int rank, world, rows_h, D, rpc, ctas;
};

// Floats of one GPU's slot in a gather half: O and LSE, padded so that every
// slot starts on a 16-byte boundary.
__host__ __device__ inline int64_t exchange_slot_floats(int rows_h, int D) {
  return ((int64_t)rows_h * (D + 1) + 3) & ~int64_t(3);
}

__device__ __forceinline__ void st_release_sys(int32_t* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kExThreads) splitkv_exchange_merge_kernel(const ExchangeArgs a) {
  __shared__ int s_target;
  __shared__ int s_ok;
  pdl_launch_dependents();
  pdl_wait();  // the partial comes from the attention launch before this one
  const int c = blockIdx.x, tid = threadIdx.x;
  const int64_t n = exchange_slot_floats(a.rows_h, a.D);  // slot stride (16-byte multiple)
  const int r0 = c * a.rpc, r1 = min(a.rows_h, r0 + a.rpc);
  if (tid == 0) {
    s_target = a.epochs[c] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const int target = s_target;
  const int half = target & 1;
  // 1. this slice of the partial into slot `rank` of every GPU's gather half
  const int o4 = (r1 - r0) * a.D / 4;  // float4s of O (D % 4 == 0, 16-byte aligned rows)
  const float4* src_o = reinterpret_cast<const float4*>(a.part + (int64_t)r0 * a.D);
  for (int p = 0; p < a.world; ++p) {
    float* dst = a.peer_gather[p] + ((int64_t)half * a.world + a.rank) * n;
    float4* dst_o = reinterpret_cast<float4*>(dst + (int64_t)r0 * a.D);
    for (int i = tid; i < o4; i += kExThreads) dst_o[i] = src_o[i];
    for (int r = r0 + tid; r < r1; r += kExThreads) dst[(int64_t)a.rows_h * a.D + r] = a.part[(int64_t)a.rows_h * a.D + r];
  }
  __syncthreads();  // every store of the slice is issued before the flags go out
  // 2. publish, then wait for every GPU's slice of the same rows
  if (tid < a.world) st_release_sys(a.peer_flags[tid] + a.rank * a.ctas + c, target);
  if (tid < a.world && tid != a.rank) {
    const int32_t* f = a.flags_local + tid * a.ctas + c;
    const long long t0 = clock64();
    for (uint32_t i = 1;; ++i) {
      if (ld_acquire_sys(f) >= target) break;
      if ((i & 255u) == 0 && clock64() - t0 > kWaitTimeoutCycles) {
        set_status(a.status, PL_ERR_TIMEOUT);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (tid == 0) a.epochs[c] = target;
  if (!s_ok) return;
  // 3. merge rows [r0, r1) from the local half, GPU order 0..world-1
  const float* g = a.peer_gather[a.rank] + (int64_t)half * a.world * n;
  for (int r = r0; r < r1; ++r) {
    float M = -INFINITY;
    for (int p = 0; p < a.world; ++p) M = fmaxf(M, __ldcg(g + p * n + (int64_t)a.rows_h * a.D + r));
    float L = 0.f;
    if (M != -INFINITY)
      for (int p = 0; p < a.world; ++p) L += expf(__ldcg(g + p * n + (int64_t)a.rows_h * a.D + r) - M);
    for (int d = tid; d < a.D; d += kExThreads) {
      float acc = 0.f;
      if (M != -INFINITY)
        for (int p = 0; p < a.world; ++p)
          acc += expf(__ldcg(g + p * n + (int64_t)a.rows_h * a.D + r) - M) * __ldcg(g + p * n + (int64_t)r * a.D + d);
      a.out[(int64_t)r * a.D + d] = f2bf(L > 0.f ? acc / L : 0.f);
    }
  }
}

}  // namespace pl

// =================================================================== host
namespace {
typedef CUresult (*MemGetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

MemGetAddressRangeFn address_range_fn() {
  static MemGetAddressRangeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<MemGetAddressRangeFn>(p);
  }
  return fn;
}
}  // namespace

extern "C" int32_t pl_ipc_handle_bytes(void) { return (int32_t)sizeof(cudaIpcMemHandle_t); }

extern "C" int32_t pl_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out) {
  if (dev_ptr == nullptr || handle_out == nullptr || offset_out == nullptr) return PL_ERR_INVALID_ARGUMENT;
  MemGetAddressRangeFn range = address_range_fn();
  if (range == nullptr) return PL_ERR_UNSUPPORTED;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return PL_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return pl_host::record_cuda_error(e);
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = (int64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return PL_OK;
}

extern "C" int32_t pl_ipc_import(const void* handle, int64_t offset, void** dev_ptr_out) {
  if (handle == nullptr || dev_ptr_out == nullptr || offset < 0) return PL_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return pl_host::record_cuda_error(e);
  *dev_ptr_out = static_cast<uint8_t*>(base) + offset;
  return PL_OK;
}

extern "C" int32_t pl_ipc_close(void* dev_ptr, int64_t offset) {
  if (dev_ptr == nullptr || offset < 0) return PL_ERR_INVALID_ARGUMENT;
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(dev_ptr) - offset);
  if (e != cudaSuccess) return pl_host::record_cuda_error(e);
  return PL_OK;
}

extern "C" int64_t pl_splitkv_exchange_slot_floats(int32_t rows_h, int32_t head_dim) {
  if (rows_h < 0 || head_dim <= 0) return 0;
  return pl::exchange_slot_floats(rows_h, head_dim);
}

extern "C" int32_t pl_splitkv_exchange_ctas(int32_t rows_h, int32_t rows_per_cta) {
  if (rows_h <= 0 || rows_per_cta <= 0) return 0;
  return (rows_h + rows_per_cta - 1) / rows_per_cta;
}

extern "C" int32_t pl_splitkv_exchange_merge(const float* part, void* const* peer_gather_dev,
                                             int32_t* const* peer_flags_dev, const int32_t* flags_local,
                                             int32_t* epochs, int32_t rank, int32_t world, int32_t rows_h,
                                             int32_t head_dim, int32_t rows_per_cta, void* out, int32_t* status_dev,
                                             void* stream) {
  if (rows_h == 0) return PL_OK;
  if (part == nullptr || peer_gather_dev == nullptr || peer_flags_dev == nullptr || flags_local == nullptr ||
      epochs == nullptr || out == nullptr || world < 2 || world > 64 || rank < 0 || rank >= world || rows_h < 0 ||
      head_dim <= 0 || rows_per_cta <= 0)
    return PL_ERR_INVALID_ARGUMENT;
  if (head_dim % 4 || (reinterpret_cast<uintptr_t>(part) & 15)) return PL_ERR_UNSUPPORTED;
  pl::ExchangeArgs a;
  a.part = part;
  a.peer_gather = reinterpret_cast<float* const*>(peer_gather_dev);
  a.peer_flags = peer_flags_dev;
  a.flags_local = flags_local;
  a.epochs = epochs;
  a.out = static_cast<pl::bf16*>(out);
  a.status = status_dev;
  a.rank = rank;
  a.world = world;
  a.rows_h = rows_h;
  a.D = head_dim;
  a.rpc = rows_per_cta;
  a.ctas = pl_splitkv_exchange_ctas(rows_h, rows_per_cta);
  return pl_host::launch_pdl(pl::splitkv_exchange_merge_kernel, dim3(a.ctas), dim3(pl::kExThreads), 0, stream, a);
}
