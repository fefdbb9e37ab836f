// exchange.cu -- exchange of attention outputs between the GPUs of a
// KV-head-sharded job (no reference counterpart; s1-infer runs one host
// thread).
//
// Every rank owns one device allocation: two layer slots of the token-major
// output [rows][all query heads][head_dim], one 64-bit word per element
// (epoch << 32 | float bits; layers alternate slots by epoch parity).  The
// allocation is shared with the other ranks' processes through CUDA IPC
// handles; the decode kernels store every finished element into its place
// in all ranks' slot (NVLink stores of whole words).  A reader polls the
// words themselves until each carries the epoch: no fence, flag or counter
// on the writer's side, and a word is never seen half written.  Reuse of a
// slot two layers later is safe because every wait checks the words of ALL
// ranks: no rank writes epoch e + 2 before it has waited for epoch e + 1,
// which every rank writes only after its own wait for epoch e, i.e. after
// it read the slot.
#include <algorithm>
#include <cstring>

#include "internal.h"

namespace s1kv {
namespace {

constexpr uint32_t kWaitSpins = 1u << 24;  // per thread: about a second with the back-off below
constexpr int kWaitThreads = 256;
constexpr int kWaitPer = 4;                 // words per thread per pass, loads in flight together

size_t alloc_bytes(int64_t slot_floats) { return (size_t)2 * slot_floats * sizeof(uint64_t); }

// Polls words [0, words) of a slot until each carries `epoch`; when dst is
// set, the words of heads [head0, head0 + n_heads) go to dst [rows]
// [n_heads][D] as floats.  A thread gives up after kWaitSpins polls in all
// and sets the timeout bit (dst is then incomplete).  Launched as a
// programmatic dependent launch that does NOT wait for the decode kernel
// before it (no griddepcontrol.wait): the words carry their epoch, so it
// polls them while the decode kernel still merges splits and pushes rows,
// and completes once every word has landed rather than when the decode
// kernel's remote stores are acknowledged.  That is safe because the
// decode kernel lets it launch only after its main loop (every kernel
// before it in the stream has completed by then), this kernel writes only
// dst, which the decode kernel never touches, and once every word is
// present the decode kernel has done all its reads and counter resets.
__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

__global__ void exchange_wait_kernel(const uint64_t* slot, int64_t words, uint32_t epoch, int* err, int heads_total,
                                     int D, int head0, int n_heads, float* dst) {
    pdl_trigger();
    uint32_t spins = 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < words; i0 += kWaitPer * stride) {
        // the pass's words are requested together (one round trip), then each
        // is polled again until its epoch matches
        uint64_t w[kWaitPer];
#pragma unroll
        for (int u = 0; u < kWaitPer; u++) w[u] = i0 + u * stride < words ? ld_word(slot + i0 + u * stride) : 0;
#pragma unroll
        for (int u = 0; u < kWaitPer; u++) {
            const int64_t i = i0 + u * stride;
            if (i >= words) break;
            while ((uint32_t)(w[u] >> 32) != epoch) {
                if (++spins >= kWaitSpins) {
                    atomicOr(err, kErrTimeout);
                    return;
                }
                __nanosleep(64);
                w[u] = ld_word(slot + i);
            }
            if (dst) {
                const int64_t rh = i / D;
                const int hh = (int)(rh % heads_total) - head0;
                if (hh >= 0 && hh < n_heads)
                    dst[((rh / heads_total) * n_heads + hh) * D + i % D] = __uint_as_float((uint32_t)w[u]);
            }
        }
    }
}

}  // namespace

// Fills the exchange fields of `ap` for a launch writing `epoch`'s slot.
int exchange_params(const s1kv_exchange* ex, uint32_t epoch, int32_t head0, int32_t heads_total, AttnParams* ap) {
    if (!ex->opened && ex->world > 1) return set_error(S1KV_EINVAL, "exchange: peers not opened");
    const size_t off = (size_t)(epoch & 1) * ex->slot_floats * sizeof(uint64_t);
    ap->xout = reinterpret_cast<uint64_t*>(ex->base + off);
    ap->out_stride = heads_total;
    ap->out_head0 = head0;
    ap->n_peers = 0;
    for (int q = 0; q < ex->world; q++)
        if (q != ex->rank) ap->xpeer[ap->n_peers++] = reinterpret_cast<uint64_t*>(ex->peer_base[q] + off);
    ap->epoch = epoch;
    return S1KV_OK;
}

// The words of the slot that `epoch`'s attention fills (rows x heads x D of
// the batch; every rank runs the same shape).
void exchange_record(s1kv_exchange* ex, uint32_t epoch, int64_t words) {
    ex->used[epoch & 1] = words;
    ex->used_epoch[epoch & 1] = epoch;
}

}  // namespace s1kv

using namespace s1kv;

extern "C" {

int s1kv_exchange_create(int device, int32_t rank, int32_t world, int64_t slot_floats, s1kv_exchange** out) {
    if (!out || world < 1 || world > 8 || rank < 0 || rank >= world || slot_floats <= 0)
        return set_error(S1KV_EINVAL, "s1kv_exchange_create: bad arguments (world 1..8)");
    *out = nullptr;
    S1KV_ON_DEVICE(device);
    auto* ex = new s1kv_exchange();
    ex->device = device;
    ex->rank = rank;
    ex->world = world;
    ex->slot_floats = slot_floats;
    cudaError_t e = cudaMalloc((void**)&ex->base, alloc_bytes(slot_floats));
    if (e == cudaSuccess) e = cudaMemset(ex->base, 0, alloc_bytes(slot_floats));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (ex->base) cudaFree(ex->base);
        delete ex;
        return cuda_error(e, "s1kv_exchange_create");
    }
    ex->d_err = device_error_word(device);
    ex->opened = world == 1;
    *out = ex;
    return S1KV_OK;
}

int s1kv_exchange_handle(const s1kv_exchange* ex, void* handle) {
    if (!ex || !handle) return set_error(S1KV_EINVAL, "null argument");
    S1KV_ON_DEVICE(ex->device);
    cudaIpcMemHandle_t h;
    S1KV_CUDA(cudaIpcGetMemHandle(&h, ex->base));
    std::memcpy(handle, &h, sizeof(h));
    return S1KV_OK;
}

int s1kv_exchange_open(s1kv_exchange* ex, const void* handles) {
    if (!ex || !handles) return set_error(S1KV_EINVAL, "null argument");
    S1KV_ON_DEVICE(ex->device);
    for (int q = 0; q < ex->world; q++) {
        if (q == ex->rank || ex->peer_base[q]) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const char*>(handles) + (size_t)q * sizeof(h), sizeof(h));
        void* ptr = nullptr;
        S1KV_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        ex->peer_base[q] = static_cast<char*>(ptr);
        ex->peer_ipc[q] = true;
    }
    ex->opened = true;
    return S1KV_OK;
}

void* s1kv_exchange_base(const s1kv_exchange* ex) { return ex ? ex->base : nullptr; }

int s1kv_exchange_open_local(s1kv_exchange* ex, void* const* bases) {
    if (!ex || !bases) return set_error(S1KV_EINVAL, "null argument");
    S1KV_ON_DEVICE(ex->device);
    for (int q = 0; q < ex->world; q++) {
        if (q == ex->rank || ex->peer_base[q]) continue;
        if (!bases[q]) return set_error(S1KV_EINVAL, "s1kv_exchange_open_local: null base of rank %d", q);
        cudaPointerAttributes a{};
        S1KV_CUDA(cudaPointerGetAttributes(&a, bases[q]));
        if (a.type != cudaMemoryTypeDevice)
            return set_error(S1KV_EINVAL, "s1kv_exchange_open_local: base of rank %d is not device memory", q);
        if (a.device != ex->device) {
            // another GPU of this process: its memory must be reachable by
            // peer access from this one
            int can = 0;
            S1KV_CUDA(cudaDeviceCanAccessPeer(&can, ex->device, a.device));
            if (!can)
                return set_error(S1KV_EINVAL, "s1kv_exchange_open_local: device %d cannot reach device %d",
                                 ex->device, a.device);
            const cudaError_t e = cudaDeviceEnablePeerAccess(a.device, 0);
            if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
            else if (e != cudaSuccess) return cuda_error(e, "cudaDeviceEnablePeerAccess");
        }
        ex->peer_base[q] = static_cast<char*>(bases[q]);
        ex->peer_ipc[q] = false;
    }
    ex->opened = true;
    return S1KV_OK;
}

void* s1kv_exchange_buffer(const s1kv_exchange* ex, uint32_t epoch) {
    if (!ex) return nullptr;
    return ex->base + (size_t)(epoch & 1) * ex->slot_floats * sizeof(uint64_t);
}

static int exchange_wait_impl(s1kv_exchange* ex, uint32_t epoch, int64_t words, int32_t heads_total, int32_t head_dim,
                              int32_t head0, int32_t n_heads, float* dst, void* stream) {
    S1KV_ON_DEVICE(ex->device);
    if (words <= 0) return S1KV_OK;
    const uint64_t* slot = static_cast<const uint64_t*>(s1kv_exchange_buffer(ex, epoch));
    const int64_t per_cta = (int64_t)kWaitThreads * kWaitPer;
    const int blocks = (int)std::min<int64_t>(4 * 148, (words + per_cta - 1) / per_cta);
    S1KV_CUDA(launch_pdl(exchange_wait_kernel, dim3(blocks), dim3(kWaitThreads), 0, (cudaStream_t)stream, slot, words, epoch,
                         ex->d_err, heads_total, head_dim, head0, n_heads, dst));
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

int s1kv_exchange_wait(s1kv_exchange* ex, uint32_t epoch, void* stream) {
    if (!ex || epoch == 0) return set_error(S1KV_EINVAL, "s1kv_exchange_wait: null exchange or epoch 0");
    // the words this rank's attention for the epoch filled; without one, the
    // whole slot
    const int64_t words = ex->used_epoch[epoch & 1] == epoch ? ex->used[epoch & 1] : ex->slot_floats;
    return exchange_wait_impl(ex, epoch, words, 1, 1, 0, 0, nullptr, stream);
}

int s1kv_exchange_wait_copy(s1kv_exchange* ex, uint32_t epoch, int32_t rows, int32_t heads_total, int32_t head_dim,
                            int32_t head0, int32_t n_heads, float* dst, void* stream) {
    const int64_t words = (int64_t)rows * heads_total * head_dim;
    if (!ex || !dst || epoch == 0 || rows < 0 || heads_total <= 0 || head_dim <= 0 || head0 < 0 || n_heads <= 0 ||
        head0 + n_heads > heads_total || words > ex->slot_floats ||
        (ex->used_epoch[epoch & 1] == epoch && ex->used[epoch & 1] != words))
        return set_error(S1KV_EINVAL, "s1kv_exchange_wait_copy: bad shape (rows x heads_total x head_dim within the "
                                      "slot and equal to what the epoch's attention wrote; epochs start at 1)");
    return exchange_wait_impl(ex, epoch, words, heads_total, head_dim, head0, n_heads, dst, stream);
}

int s1kv_exchange_destroy(s1kv_exchange* ex) {
    if (!ex) return S1KV_OK;
    DeviceGuard guard(ex->device);
    cudaDeviceSynchronize();
    for (int q = 0; q < ex->world; q++)
        if (ex->peer_base[q] && ex->peer_ipc[q]) cudaIpcCloseMemHandle(ex->peer_base[q]);
    if (ex->base) cudaFree(ex->base);
    delete ex;
    return S1KV_OK;
}

}  // extern "C"
