// attn_noalloc.cu — sj_attn_noalloc: scheduled attention that allocates nothing.
//
// Who needs it: callers that cannot call cudaMalloc at all — a host process
// whose device memory is owned by its own pool allocator (the runtime may
// refuse or fragment it), or an embedding that forbids allocation on its
// inference path.  The engine's attention launch needs a scratch buffer (the
// query-tile schedule, longest sequences first), which the engine allocates
// once.  This entry point keeps that scratch in a file-scope static device
// array instead, so a call allocates no device memory and needs no workspace
// from the caller; inputs and outputs are still the caller's buffers.
//
// Limits and rules:
//  * at most kSchedMax (65536) query tiles per call — tiles of 128 rows with
//    head_dim 64, of 64 rows otherwise; larger batches are rejected with
//    SJ_ERR_INVALID and a message;
//  * the array is one per GPU that loads the library and stays resident
//    (512 KiB) until the process exits;
//  * the first call on a device looks the array's device address up
//    (cudaGetSymbolAddress, with that device current); make that first call
//    before any stream capture;
//  * every call writes the whole schedule it uses (nothing carries over), but
//    calls share the one array: calls whose launches overlap on the GPU (two
//    streams, two host threads) race on it — serialise them;
//  * failures inside the kernels (a bounded wait that ran out, device
//    cu_seqlens that disagree with the host mirror) are reported by
//    sj_check_device_errors, which reads file-scope status words: that check
//    allocates nothing either.
#include <mutex>
#include <string>

#include "../../include/snapjudge_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace sjb {
namespace {

constexpr int kSchedMax = 65536;
constexpr int kBuckets = 256;  // sequences bucketed by their tile count (capped)

// The schedule scratch: (segment, first query row) per tile.
static __device__ __align__(256) int2 g_sched_scratch[kSchedMax];
// Set by build_schedule when the device cu_seqlens give another tile count
// than the host mirror did (read and cleared by sj_check_device_errors).
static __device__ int g_sched_err;

// Longest-first query-tile schedule of B segments, built by one block:
// tiles of segments with more tiles come first (bucketed counting sort).
// n_tiles (<= kSchedMax) is the count the host found in its mirror of cu; the
// kernel writes exactly entries [0, n_tiles).  If the device array disagrees,
// every entry becomes an idle tile (first row past any segment, which the
// attention kernel skips), g_sched_err is set and nothing past n_tiles is
// written.
__global__ void __launch_bounds__(1024) build_schedule(const int32_t* __restrict__ cu, int B,
                                                       int qt, int n_tiles,
                                                       int2* __restrict__ sched) {
  __shared__ int count[kBuckets];
  __shared__ int cursor[kBuckets];
  __shared__ int total;
  for (int i = threadIdx.x; i < kBuckets; i += blockDim.x) count[i] = 0;
  if (threadIdx.x == 0) total = 0;
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int n = cu[b + 1] - cu[b];
    const int nt = n > 0 ? (n + qt - 1) / qt : 0;
    if (nt > 0) {
      atomicAdd(&count[min(nt, kBuckets - 1)], nt);
      atomicAdd(&total, nt);
    }
  }
  __syncthreads();
  if (total != n_tiles) {  // device cu_seqlens differ from the host mirror
    for (int t = threadIdx.x; t < n_tiles; t += blockDim.x) sched[t] = make_int2(0, 0x3fffffff);
    if (threadIdx.x == 0) g_sched_err = 1;
    return;
  }
  if (threadIdx.x == 0) {  // bucket start offsets, most tiles first
    int off = 0;
    for (int k = kBuckets - 1; k >= 1; --k) {
      cursor[k] = off;
      off += count[k];
    }
  }
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int n = cu[b + 1] - cu[b];
    const int nt = n > 0 ? (n + qt - 1) / qt : 0;
    if (nt == 0) continue;
    const int at = atomicAdd(&cursor[min(nt, kBuckets - 1)], nt);
    for (int t = 0; t < nt && at + t < n_tiles; ++t) sched[at + t] = make_int2(b, t * qt);
  }
}

std::mutex g_mu;
int2* g_sched_ptr[64] = {};  // device address of g_sched_scratch, per device ordinal

int fail(int code, const std::string& m) {
  set_last_error(m);
  return code;
}

}  // namespace

cudaError_t attn_noalloc_take_status(int* code) {
  int v = 0;
  cudaError_t rc = cudaMemcpyFromSymbol(&v, g_sched_err, sizeof(int));
  if (rc == cudaSuccess && v != 0) {
    const int zero = 0;
    rc = cudaMemcpyToSymbol(g_sched_err, &zero, sizeof(int));
  }
  *code = v;
  return rc;
}

}  // namespace sjb

extern "C" {

int sj_attn_noalloc(const sj_bf16* qkv, const int32_t* cu_seqlens, const int32_t* cu_seqlens_host,
                    const int32_t* kv_lens, sj_bf16* O, int B, int H, int Dh, int window,
                    void* stream) {
  using namespace sjb;
  if (!cu_seqlens_host) return fail(SJ_ERR_INVALID, "cu_seqlens_host is null");
  if (B < 0 || H <= 0 || window < 0) return fail(SJ_ERR_INVALID, "bad attention shape");
  if (B > 0 && cu_seqlens_host[0] != 0) return fail(SJ_ERR_INVALID, "cu_seqlens[0] must be 0");
  const bool tc = attn_tc_supported(Dh);
  if (!tc && Dh != 8 && Dh != 16 && Dh != 32 && Dh != 128)
    return fail(SJ_ERR_UNSUPPORTED, "head_dim must be 8, 16, 32, 64 or 128");
  const int qt = tc ? 128 : 64;
  long long tiles = 0;
  for (int b = 0; b < B; ++b) {
    const int n = cu_seqlens_host[b + 1] - cu_seqlens_host[b];
    if (n < 0) return fail(SJ_ERR_INVALID, "cu_seqlens must be non-decreasing");
    tiles += (n + qt - 1) / qt;
  }
  if (tiles > kSchedMax)
    return fail(SJ_ERR_INVALID, "sj_attn_noalloc: " + std::to_string(tiles) +
                                    " query tiles exceed the static schedule capacity of " +
                                    std::to_string(kSchedMax) + " (split the batch)");
  const int T = B > 0 ? cu_seqlens_host[B] : 0;
  if (tiles == 0 || T == 0) return SJ_OK;
  if (!qkv || !O || !cu_seqlens) return fail(SJ_ERR_INVALID, "null attention operand");
  int dev = 0;
  cudaError_t rc = cudaGetDevice(&dev);
  if (rc != cudaSuccess)
    return fail(SJ_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(rc));
  if (dev < 0 || dev >= 64)
    return fail(SJ_ERR_UNSUPPORTED, "sj_attn_noalloc: device ordinal " + std::to_string(dev) +
                                        " >= 64 (the library keeps the array's address for "
                                        "ordinals 0-63)");
  int2* sched = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_sched_ptr[dev]) {  // once per device, with that device current
      rc = cudaGetSymbolAddress(reinterpret_cast<void**>(&g_sched_ptr[dev]), g_sched_scratch);
      if (rc != cudaSuccess) {
        g_sched_ptr[dev] = nullptr;
        return fail(SJ_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(rc));
      }
    }
    sched = g_sched_ptr[dev];
  }
  auto st = static_cast<cudaStream_t>(stream);
  build_schedule<<<1, 1024, 0, st>>>(cu_seqlens, B, qt, (int)tiles, sched);
  if ((rc = cudaGetLastError()) != cudaSuccess)
    return fail(SJ_ERR_CUDA, std::string("build_schedule: ") + cudaGetErrorString(rc));
  const bf16* q = reinterpret_cast<const bf16*>(qkv);
  bf16* o = reinterpret_cast<bf16*>(O);
  rc = tc ? attn_tc(q, cu_seqlens, kv_lens, o, T, H, window, sched, (int)tiles, B, 0, nullptr, st)
          : attn_simt<bf16>(q, cu_seqlens, kv_lens, o, H, Dh, window, sched, (int)tiles, B, 0, st);
  if (rc != cudaSuccess)
    return fail(SJ_ERR_CUDA, std::string("attention: ") + cudaGetErrorString(rc));
  return SJ_OK;
}

}  // extern "C"
