// shim_internal.h -- helpers shared by the shim's source files.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>

class KVBlockPool;

namespace s1kv_shim {

// Throws std::runtime_error with the engine's last error message.
[[noreturn]] void raise(int status, const char* what);
void check(int status, const char* what);
void cuda_check(cudaError_t e, const char* what);

// Device storage address -> owning pool, for KVView lookups.
void register_pool(const void* base, const KVBlockPool* pool);
const KVBlockPool* pool_of(const void* base);

// Reused per-thread device staging buffer.
struct DeviceBuffer {
    void* p = nullptr;
    size_t cap = 0;
    ~DeviceBuffer();
    void* get(size_t bytes);
};

}  // namespace s1kv_shim
