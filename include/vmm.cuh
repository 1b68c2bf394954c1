#pragma once
// VMM helpers of the harness API (include/vmm.cuh:5-38 of the reference), on
// top of libagg.so.  Same names and signatures; vm_set_access is added because
// a mapping made by vm_map alone cannot be touched until access is granted.
#include <cuda.h>

#include "agg.h"
#include "util.cuh"

static constexpr CUmemAllocationHandleType HANDLE_TYPE = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
typedef CUmemGenericAllocationHandle handle;

namespace agg_detail {
inline void die(const char* what) {
    std::fprintf(stderr, "%s: %s\n", what, agg_last_error());
    std::exit(EXIT_FAILURE);
}
}  // namespace agg_detail

// Physical allocation of at least `size` bytes on `device_id`, rounded up to the
// allocation granularity (the rounded size is written to *allocated_size).
__host__ inline static void vm_alloc(handle* h, size_t* allocated_size, const size_t size, const int device_id) {
    uint64_t raw = 0;
    if (agg_vm_alloc(&raw, allocated_size, size, device_id) != AGG_OK) agg_detail::die("vm_alloc");
    *h = static_cast<handle>(raw);
}

// Reserve a VA range of `size` bytes and map the allocation there.
__host__ inline static void vm_map(void** ptr, const handle& h, const size_t size) {
    uint64_t va = 0;
    if (agg_vm_map(&va, static_cast<uint64_t>(h), size) != AGG_OK) agg_detail::die("vm_map");
    *ptr = reinterpret_cast<void*>(va);
}

// Grant read/write access to the mapping for every listed device.
__host__ inline static void vm_set_access(void* ptr, const size_t size, const int* devices, int ndevices) {
    if (agg_vm_set_access(reinterpret_cast<uint64_t>(ptr), size, devices, ndevices) != AGG_OK)
        agg_detail::die("vm_set_access");
}

__host__ inline static void vm_unmap(void* ptr, const size_t size) {
    if (agg_vm_unmap_free(reinterpret_cast<uint64_t>(ptr), size) != AGG_OK) agg_detail::die("vm_unmap");
}

__host__ inline static void vm_free(const handle& h) {
    if (agg_vm_release(static_cast<uint64_t>(h)) != AGG_OK) agg_detail::die("vm_free");
}
