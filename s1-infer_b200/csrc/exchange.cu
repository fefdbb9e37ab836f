// exchange.cu -- exchange of attention outputs between the GPUs of a
// KV-head-sharded job (no reference counterpart; s1-infer runs one host
// thread).
//
// Every rank owns one device allocation: two layer slots of the token-major
// output [rows][all query heads][head_dim] (fp32; layers alternate slots),
// then flags[2][8] (uint32, the epoch rank r last finished in that slot),
// then one completion counter.  The allocation is shared with the other
// ranks' processes through CUDA IPC handles; the decode kernels store every
// finished row into its place in all ranks' slot (NVLink stores), and the
// launch's last CTA sets this rank's flag on every rank (release, system
// scope).  Before reading a slot, a rank waits (bounded) until every rank's
// flag reached the epoch.  Reuse of a slot two layers later is safe: no rank
// can reach it before every rank has finished the layer in between, which
// needs this slot's contents.
#include <cstring>

#include "internal.h"

namespace s1kv {
namespace {

constexpr uint32_t kWaitSpins = 1u << 24;  // about a second with the back-off below

size_t flags_offset(int64_t slot_floats) { return (size_t)2 * slot_floats * sizeof(float); }
size_t done_offset(int64_t slot_floats) { return flags_offset(slot_floats) + 2 * 8 * sizeof(uint32_t); }
size_t alloc_bytes(int64_t slot_floats) { return done_offset(slot_floats) + 256; }

// Lane r of warp 0 waits until rank r's flag in this slot has reached
// `epoch`; then, when `dst` is set, the CTA copies heads [head0, head0 +
// n_heads) of every row of the slot [rows][heads_total][D] into dst [rows]
// [n_heads][D].  Launched as a programmatic dependent launch: the CTA may
// become resident while this rank's decode kernel still runs, and waits for
// it to complete (griddepcontrol.wait) before polling, so the only waits
// left are on the other GPUs' kernels.
__global__ void exchange_wait_kernel(const uint32_t* flags, int world, uint32_t epoch, int* err, const float* slot,
                                     int rows, int heads_total, int D, int head0, int n_heads, float* dst) {
    pdl_enter();
    __shared__ int ok;
    if (threadIdx.x < 32) {
        const int r = threadIdx.x;
        bool seen = r >= world;
        for (uint32_t i = 0; i < kWaitSpins && !seen; i++) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + r) : "memory");
            seen = (int32_t)(v - epoch) >= 0;
            if (!seen) __nanosleep(64);
        }
        const bool all = __all_sync(0xffffffffu, seen);
        if (threadIdx.x == 0) {
            if (!all) atomicOr(err, kErrTimeout);
            ok = all;
        }
    }
    __syncthreads();
    if (!dst || !ok) return;
    const int per_row = n_heads * D / 4;  // float4 per row
    for (int i = threadIdx.x; i < rows * per_row; i += blockDim.x) {
        const int row = i / per_row, c = i % per_row;
        reinterpret_cast<float4*>(dst)[i] =
            reinterpret_cast<const float4*>(slot + ((int64_t)row * heads_total + head0) * D)[c];
    }
}

}  // namespace

// Fills the exchange fields of `ap` for a launch writing `epoch`'s slot.
int exchange_params(const s1kv_exchange* ex, uint32_t epoch, int32_t head0, int32_t heads_total, AttnParams* ap) {
    if (!ex->opened && ex->world > 1) return set_error(S1KV_EINVAL, "exchange: peers not opened");
    const int s = epoch & 1;
    ap->out = reinterpret_cast<float*>(ex->base + (size_t)s * ex->slot_floats * sizeof(float));
    ap->out_stride = heads_total;
    ap->out_head0 = head0;
    ap->n_peers = 0;
    for (int q = 0; q < ex->world; q++) {
        char* b = q == ex->rank ? ex->base : ex->peer_base[q];
        if (q != ex->rank) ap->peer_out[ap->n_peers++] = reinterpret_cast<float*>(b + (size_t)s * ex->slot_floats * sizeof(float));
        ap->flag_dst[q] = reinterpret_cast<uint32_t*>(b + flags_offset(ex->slot_floats)) + s * 8 + ex->rank;
    }
    ap->n_flags = ex->world;
    ap->done = reinterpret_cast<uint32_t*>(ex->base + done_offset(ex->slot_floats));
    ap->epoch = epoch;
    return S1KV_OK;
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

float* s1kv_exchange_buffer(const s1kv_exchange* ex, uint32_t epoch) {
    if (!ex) return nullptr;
    return reinterpret_cast<float*>(ex->base + (size_t)(epoch & 1) * ex->slot_floats * sizeof(float));
}

static int exchange_wait_impl(s1kv_exchange* ex, uint32_t epoch, int32_t rows, int32_t heads_total, int32_t head_dim,
                              int32_t head0, int32_t n_heads, float* dst, void* stream) {
    if (!ex) return set_error(S1KV_EINVAL, "null exchange");
    S1KV_ON_DEVICE(ex->device);
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(ex->base + flags_offset(ex->slot_floats)) + (epoch & 1) * 8;
    const float* slot = reinterpret_cast<const float*>(ex->base + (size_t)(epoch & 1) * ex->slot_floats * sizeof(float));
    S1KV_CUDA(launch_pdl(exchange_wait_kernel, dim3(1), dim3(dst ? 256 : 32), 0, (cudaStream_t)stream, flags, ex->world,
                         epoch, ex->d_err, slot, rows, heads_total, head_dim, head0, n_heads, dst));
    g_launches++;
    S1KV_CUDA(cudaGetLastError());
    return S1KV_OK;
}

int s1kv_exchange_wait(s1kv_exchange* ex, uint32_t epoch, void* stream) {
    return exchange_wait_impl(ex, epoch, 0, 0, 0, 0, 0, nullptr, stream);
}

int s1kv_exchange_wait_copy(s1kv_exchange* ex, uint32_t epoch, int32_t rows, int32_t heads_total, int32_t head_dim,
                            int32_t head0, int32_t n_heads, float* dst, void* stream) {
    if (!ex || !dst || rows < 0 || heads_total <= 0 || head_dim <= 0 || head0 < 0 || n_heads <= 0 ||
        head0 + n_heads > heads_total || (n_heads * head_dim) % 4 || head_dim % 4 ||
        (int64_t)rows * heads_total * head_dim > ex->slot_floats || ((uintptr_t)dst & 15))
        return set_error(S1KV_EINVAL, "s1kv_exchange_wait_copy: bad shape (head_dim a multiple of 4, dst 16-byte "
                                      "aligned, rows x heads_total x head_dim within the slot)");
    return exchange_wait_impl(ex, epoch, rows, heads_total, head_dim, head0, n_heads, dst, stream);
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
