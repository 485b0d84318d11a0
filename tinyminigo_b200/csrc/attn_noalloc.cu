// Decode attention that allocates nothing (tmg_op_attn_decode_noalloc).
//
// Why: the regular op entry point grows a per-context scratch buffer with
// cudaMalloc the first time it needs one.  Some callers cannot allocate at
// the moment they run attention:
//  * a serving loop that hands out its whole device-memory budget at
//    start-up and must not grow afterwards (an allocation there can fail or
//    push a neighbour out of memory);
//  * an engine that owns the GPU's memory through its own pool or arena and
//    forbids allocations behind its back (device memory it did not hand
//    out is memory it cannot account for);
//  * a latency-bound path that cannot afford the device-wide
//    synchronization an allocation or free implies.
// This variant takes its split-KV partials, the per-head tickets and the
// query position from one file-scope __device__ array per device, whose
// address is looked up once per device and reused.
//
// Limits and rules:
//  * kScratchBytes (4 MiB) bounds the partials; larger requests are rejected
//    before anything is enqueued.
//  * The first call on a device does the setup (cudaGetSymbolAddress, which
//    also loads this module); make it before any stream capture.  Only a
//    successful lookup is kept: a failed one is tried again on the next
//    call.  The address belongs to the device's primary context (the one
//    the CUDA runtime uses), for the life of the process.
//  * The tickets must be zero when the attention kernel starts: static
//    storage starts zeroed, the kernel's last split of each head resets its
//    ticket, and every call also zeroes them (with the position word) in a
//    one-thread-block kernel on the same stream just before the attention
//    launch.
//  * There is one scratch per device: calls that overlap on one device (two
//    streams, two threads, two contexts) race on it.  Order them.
#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.cuh"

namespace tmg {

namespace {

constexpr size_t kScratchBytes = size_t(4) << 20;
constexpr size_t kHeaderBytes = 4096;  // [0] position word, [16..] tickets
constexpr int kTicketWord = 16;
constexpr int kMaxTickets = int(kHeaderBytes / 4) - kTicketWord;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

std::mutex g_mu[kMaxDevices];
void* g_addr[kMaxDevices];  // non-null once the lookup on that device succeeded

// The scratch address on `device`, which must be the current device.
cudaError_t scratch_on(int device, unsigned char** out) {
  std::lock_guard<std::mutex> lk(g_mu[device]);
  if (!g_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return e;
    g_addr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_addr[device]);
  return cudaSuccess;
}

// The per-call state the attention kernel expects at its start: the query
// position word and zeroed tickets.
__global__ void noalloc_prep_kernel(int32_t* pos, unsigned int* tickets, int n, int32_t pos_value) {
  if (threadIdx.x == 0) *pos = pos_value;
  for (int i = threadIdx.x; i < n; i += blockDim.x) tickets[i] = 0u;
}

}  // namespace

int attn_decode_noalloc(int device, int num_sms, cudaStream_t s, const float* q, const float* keys,
                        const float* values, int64_t n_ctx, int n_q, int n_kv, int head_dim,
                        float* out, std::string* why) {
  if (device < 0 || device >= kMaxDevices) {
    *why = "device index beyond the static scratch table";
    return 1;
  }
  const int G = n_q / n_kv;
  const int nsplit = attn_decode_nsplit(n_kv, 1, n_ctx, num_sms);
  if (!attn_decode_shape_ok(n_q, n_kv, head_dim, n_ctx, nsplit, why)) return 1;
  const size_t part_bytes = size_t(n_kv) * nsplit * G * (head_dim + 2) * sizeof(float);
  if (n_kv > kMaxTickets || part_bytes > kScratchBytes - kHeaderBytes) {
    *why = "needs " + std::to_string(part_bytes + kHeaderBytes) + " bytes of scratch (" +
           std::to_string(n_kv) + " kv heads); the static scratch holds " +
           std::to_string(kScratchBytes) + " bytes and " + std::to_string(kMaxTickets) + " heads";
    return 2;
  }
  unsigned char* base = nullptr;
  cudaError_t e = scratch_on(device, &base);
  if (e != cudaSuccess) {
    *why = std::string("scratch setup: ") + cudaGetErrorString(e);
    return 3;
  }
  int32_t* posw = reinterpret_cast<int32_t*>(base);
  unsigned int* tickets = reinterpret_cast<unsigned int*>(base) + kTicketWord;
  noalloc_prep_kernel<<<1, 128, 0, s>>>(posw, tickets, n_kv, int32_t(n_ctx - 1));
  e = cudaGetLastError();
  if (e == cudaSuccess) {
    AttnDecodeArgs a;
    a.qkv = q;
    a.qkv_ld = 0;
    a.kc = const_cast<float*>(keys);
    a.vc = const_cast<float*>(values);
    a.cap = n_ctx;
    a.out = out;
    a.part = reinterpret_cast<float*>(base + kHeaderBytes);
    a.ticket = tickets;
    a.pos_override = posw;
    a.nq = n_q;
    a.nkv = n_kv;
    a.d = head_dim;
    a.nsplit = nsplit;
    a.M = 1;
    a.scale = 1.0f / sqrtf(float(head_dim));
    e = launch_attn_decode(a, s, false);
  }
  if (e != cudaSuccess) {
    *why = std::string("attention: ") + cudaGetErrorString(e);
    return 3;
  }
  return 0;
}

}  // namespace tmg
