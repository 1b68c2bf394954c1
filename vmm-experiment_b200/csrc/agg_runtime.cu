// Host runtime of libagg.so: driver entry points, error reporting, the VMM
// helpers and the two ways of bringing up the NVLink multicast slab.
//
//  * One process, one thread per GPU — the reference's model
//    (minfer_spmm_init, vmm/multimem.cu:74-101): the first caller creates the
//    multicast object for devices 0..world-1 and adds them all (create_mc,
//    vmm/multimem.cu:11-40); every rank then creates its physical slab, binds it
//    to the multicast object and maps a unicast VA readable by all GPUs plus the
//    multicast VA (rank_setup, vmm/multimem.cu:42-72).
//
//  * One process per GPU (torch.distributed, MPI, ...) — no counterpart in the
//    reference: the same handles are exported as POSIX file descriptors and
//    passed between the processes with SCM_RIGHTS over abstract unix sockets.
//
// Slab layout: gathered data from offset 0, the flag area at `flag_off`
// (320 MiB inside the reference's 512 MiB slab, include/multimem.cuh:8-9; past
// the data when the caller asks for more than 320 MiB).
#include <cuda.h>
#include <cuda_runtime.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "agg.h"
#include "agg_internal.h"

namespace agg {

// ---------------------------------------------------------------- errors
namespace {
thread_local std::string t_last_error;
}

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int check_rt(cudaError_t e, const char* what) {
    return fail(AGG_ECUDA, "%s -> %s", what, cudaGetErrorString(e));
}

int check_drv(CUresult r, const char* what) {
    const char* s = nullptr;
    const DriverApi& d = driver();
    if (d.ok && d.cuGetErrorString) d.cuGetErrorString(r, &s);
    return fail(AGG_EDRIVER, "%s -> %s (%d)", what, s ? s : "?", static_cast<int>(r));
}

// ---------------------------------------------------------------- driver table
const DriverApi& driver() {
    static DriverApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e != cudaSuccess) {
            api.why = std::string("no usable CUDA device: ") + cudaGetErrorString(e);
            return;
        }
        bool all = true;
#define AGG_LOAD_PFN(name)                                                                   \
    {                                                                                        \
        void* fn = nullptr;                                                                  \
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;              \
        cudaError_t le = cudaGetDriverEntryPointByVersion(#name, &fn, CUDART_VERSION, cudaEnableDefault, &q); \
        if (le != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {                  \
            all = false;                                                                     \
            api.why += std::string(" missing ") + #name;                                     \
        } else {                                                                             \
            api.name = reinterpret_cast<decltype(api.name)>(fn);                             \
        }                                                                                    \
    }
        AGG_DRIVER_FUNCS(AGG_LOAD_PFN)
#undef AGG_LOAD_PFN
        api.ok = all;
        if (all && api.cuInit(0) != CUDA_SUCCESS) {
            api.ok = false;
            api.why = "cuInit failed";
        }
    });
    return api;
}

namespace {

#define DRV_OR_FAIL()                                                                  \
    const DriverApi& D = driver();                                                     \
    if (!D.ok) return fail(AGG_EDRIVER, "CUDA driver unavailable:%s", D.why.c_str());

size_t round_up(size_t x, size_t g) { return (x + g - 1) / g * g; }

// Makes `device`'s primary context current for the driver calls of one entry
// point and restores the caller's device afterwards.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int device) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = cudaSetDevice(device) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

CUmemAllocationProp phys_prop(int device) {
    CUmemAllocationProp ap;
    std::memset(&ap, 0, sizeof(ap));
    ap.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    ap.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    ap.location.id = device;
    ap.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    return ap;
}

// Slab geometry for a request of `data_bytes`: the reference's 512 MiB slab with
// flags at 320 MiB when the data fits below them, otherwise flags right after
// the data (2 MiB aligned) and the slab rounded up to the multicast granularity.
void slab_geometry(size_t data_bytes, size_t gran, size_t* slab, size_t* flag_off) {
    const size_t kRefSlab = 512ull << 20, kRefFlagOff = 320ull << 20;
    if (data_bytes <= kRefFlagOff) {
        *flag_off = kRefFlagOff;
        *slab = round_up(kRefSlab, gran);
    } else {
        *flag_off = round_up(data_bytes, 2ull << 20);
        *slab = round_up(*flag_off + AGG_FLAG_BYTES, gran);
    }
}

int check_multicast_supported(int device) {
    DRV_OR_FAIL();
    CUdevice dev;
    AGG_DRV(D.cuDeviceGet(&dev, device));
    int ok = 0;
    AGG_DRV(D.cuDeviceGetAttribute(&ok, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev));
    if (!ok) return fail(AGG_ENOMULTICAST, "GPU %d has no multicast support", device);
    return AGG_OK;
}

int multicast_granularity(int world, size_t size, size_t* gran) {
    DRV_OR_FAIL();
    CUmulticastObjectProp mp;
    std::memset(&mp, 0, sizeof(mp));
    mp.numDevices = static_cast<unsigned>(world);
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    mp.size = size;
    AGG_DRV(D.cuMulticastGetGranularity(gran, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED));
    size_t g2 = 0;
    CUmemAllocationProp ap = phys_prop(0);
    AGG_DRV(D.cuMemGetAllocationGranularity(&g2, &ap, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED));
    if (g2 > *gran) *gran = g2;
    return AGG_OK;
}

int map_range(CUdeviceptr* va, size_t size, CUmemGenericAllocationHandle h, const int* devs, int ndev) {
    DRV_OR_FAIL();
    AGG_DRV(D.cuMemAddressReserve(va, size, 0, 0, 0));
    CUresult r = D.cuMemMap(*va, size, 0, h, 0);
    if (r != CUDA_SUCCESS) {
        D.cuMemAddressFree(*va, size);
        *va = 0;
        return check_drv(r, "cuMemMap");
    }
    std::vector<CUmemAccessDesc> ad(ndev);
    for (int i = 0; i < ndev; ++i) {
        std::memset(&ad[i], 0, sizeof(ad[i]));
        ad[i].location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        ad[i].location.id = devs[i];
        ad[i].flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    }
    r = D.cuMemSetAccess(*va, size, ad.data(), ndev);
    if (r != CUDA_SUCCESS) {
        D.cuMemUnmap(*va, size);
        D.cuMemAddressFree(*va, size);
        *va = 0;
        return check_drv(r, "cuMemSetAccess");
    }
    return AGG_OK;
}

void unmap_range(CUdeviceptr va, size_t size) {
    const DriverApi& D = driver();
    if (!D.ok || !va) return;
    D.cuMemUnmap(va, size);
    D.cuMemAddressFree(va, size);
}

int zero_flags(CUdeviceptr uc, size_t flag_off, int device) {
    int prev = 0;
    AGG_RT(cudaGetDevice(&prev));
    AGG_RT(cudaSetDevice(device));
    cudaError_t e = cudaMemset(reinterpret_cast<void*>(uc + flag_off), 0, AGG_FLAG_BYTES);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaSetDevice(prev);
    if (e != cudaSuccess) return check_rt(e, "zero flag area");
    return AGG_OK;
}

// ---------------------------------------------------------------- in-process mode
struct ProcessState {
    std::once_flag once;
    int world = 0;
    int rc = AGG_ESTATE;
    std::string err;
    CUmemGenericAllocationHandle mc = 0;
    size_t slab = 0, flag_off = 0;
    std::atomic<int> live{0};
};
ProcessState g_proc;

struct RankSlot {
    std::mutex mu;
    bool mapped = false;
    CUmemGenericAllocationHandle phys = 0;
    CUdeviceptr uc = 0, mc = 0;
};
RankSlot g_slots[AGG_MAX_RANKS];

int create_mc_all(int world, size_t data_bytes) {
    DRV_OR_FAIL();
    for (int d = 0; d < world; ++d) {
        int rc = check_multicast_supported(d);
        if (rc) return rc;
    }
    size_t gran = 0;
    int rc = multicast_granularity(world, 512ull << 20, &gran);
    if (rc) return rc;
    slab_geometry(data_bytes, gran, &g_proc.slab, &g_proc.flag_off);
    CUmulticastObjectProp mp;
    std::memset(&mp, 0, sizeof(mp));
    mp.numDevices = static_cast<unsigned>(world);
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    mp.size = g_proc.slab;
    AGG_DRV(D.cuMulticastCreate(&g_proc.mc, &mp));
    for (int d = 0; d < world; ++d) {
        CUdevice dev;
        AGG_DRV(D.cuDeviceGet(&dev, d));
        AGG_DRV(D.cuMulticastAddDevice(g_proc.mc, dev));
    }
    return AGG_OK;
}

void fill_info(agg_rank_info* out, int rank, int world, int device, CUdeviceptr uc, CUdeviceptr mc,
               const CUdeviceptr* peers, size_t slab, size_t flag_off) {
    if (!out) return;
    std::memset(out, 0, sizeof(*out));
    out->uc = uc;
    out->mc = mc;
    for (int i = 0; i < world && i < AGG_MAX_RANKS; ++i) out->peer_uc[i] = peers ? peers[i] : 0;
    out->slab_bytes = slab;
    out->flag_off = flag_off;
    out->rank = rank;
    out->world = world;
    out->device = device;
}

}  // namespace

// ---------------------------------------------------------------- multi-process mode
}  // namespace agg

struct agg_mp_ctx {
    int rank = 0, world = 0, device = 0;
    std::string job;
    size_t slab = 0, flag_off = 0;
    int listen_fd = -1;
    int mc_fd = -1;                                  // rank 0: exported; others: received
    int phys_fd[AGG_MAX_RANKS];                      // own exported / peers' received
    CUmemGenericAllocationHandle mc = 0;
    CUmemGenericAllocationHandle phys = 0;
    CUmemGenericAllocationHandle peer_phys[AGG_MAX_RANKS];
    CUdeviceptr uc = 0, mcva = 0;
    CUdeviceptr peer_uc[AGG_MAX_RANKS];
    bool exchanged = false, added = false, bound = false;
};

namespace agg {
namespace {

std::string sock_name(const std::string& job, int rank) {
    return "agg-" + job + "-" + std::to_string(rank);
}

int make_addr(const std::string& name, sockaddr_un* a, socklen_t* len) {
    std::memset(a, 0, sizeof(*a));
    a->sun_family = AF_UNIX;
    if (name.size() + 1 >= sizeof(a->sun_path)) return fail(AGG_EINVAL, "job id too long");
    // abstract namespace: leading NUL, no file on disk
    std::memcpy(a->sun_path + 1, name.data(), name.size());
    *len = static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + name.size());
    return AGG_OK;
}

// Message: {sender rank, number of fds}; the fds ride along as SCM_RIGHTS.
int send_fds(const std::string& to, int from_rank, const int* fds, int nfds) {
    int s = socket(AF_UNIX, SOCK_STREAM, 0);
    if (s < 0) return fail(AGG_ESYS, "socket: %s", strerror(errno));
    sockaddr_un a;
    socklen_t len = 0;
    int rc = make_addr(to, &a, &len);
    if (rc) {
        close(s);
        return rc;
    }
    int tries = 0;
    while (connect(s, reinterpret_cast<sockaddr*>(&a), len) != 0) {
        if (++tries > 2000 || (errno != ECONNREFUSED && errno != EAGAIN && errno != ENOENT)) {
            int e = errno;
            close(s);
            return fail(AGG_ESYS, "connect %s: %s", to.c_str(), strerror(e));
        }
        usleep(5000);
    }
    int32_t hdr[2] = {from_rank, nfds};
    iovec iov{hdr, sizeof(hdr)};
    char cbuf[CMSG_SPACE(sizeof(int) * 4)];
    std::memset(cbuf, 0, sizeof(cbuf));
    msghdr m;
    std::memset(&m, 0, sizeof(m));
    m.msg_iov = &iov;
    m.msg_iovlen = 1;
    if (nfds > 0) {
        m.msg_control = cbuf;
        m.msg_controllen = CMSG_SPACE(sizeof(int) * nfds);
        cmsghdr* c = CMSG_FIRSTHDR(&m);
        c->cmsg_level = SOL_SOCKET;
        c->cmsg_type = SCM_RIGHTS;
        c->cmsg_len = CMSG_LEN(sizeof(int) * nfds);
        std::memcpy(CMSG_DATA(c), fds, sizeof(int) * nfds);
    }
    ssize_t n = sendmsg(s, &m, 0);
    int e = errno;
    close(s);
    if (n != static_cast<ssize_t>(sizeof(hdr))) return fail(AGG_ESYS, "sendmsg: %s", strerror(e));
    return AGG_OK;
}

int recv_fds(int listen_fd, int* from_rank, int* fds, int* nfds) {
    int c = accept(listen_fd, nullptr, nullptr);
    if (c < 0) return fail(AGG_ESYS, "accept: %s", strerror(errno));
    int32_t hdr[2] = {-1, 0};
    iovec iov{hdr, sizeof(hdr)};
    char cbuf[CMSG_SPACE(sizeof(int) * 4)];
    msghdr m;
    std::memset(&m, 0, sizeof(m));
    m.msg_iov = &iov;
    m.msg_iovlen = 1;
    m.msg_control = cbuf;
    m.msg_controllen = sizeof(cbuf);
    ssize_t n = recvmsg(c, &m, 0);
    int e = errno;
    close(c);
    if (n != static_cast<ssize_t>(sizeof(hdr))) return fail(AGG_ESYS, "recvmsg: %s", strerror(e));
    *from_rank = hdr[0];
    *nfds = 0;
    for (cmsghdr* h = CMSG_FIRSTHDR(&m); h; h = CMSG_NXTHDR(&m, h)) {
        if (h->cmsg_level == SOL_SOCKET && h->cmsg_type == SCM_RIGHTS) {
            int k = static_cast<int>((h->cmsg_len - CMSG_LEN(0)) / sizeof(int));
            if (k > 4) k = 4;
            std::memcpy(fds, CMSG_DATA(h), sizeof(int) * k);
            *nfds = k;
        }
    }
    if (*nfds != hdr[1]) return fail(AGG_ESYS, "fd count mismatch (%d vs %d)", *nfds, hdr[1]);
    return AGG_OK;
}

}  // namespace
}  // namespace agg

using namespace agg;

extern "C" {

int agg_version(void) { return 100; }

int agg_abi_sizes(size_t* args_bytes, size_t* rank_info_bytes) {
    if (args_bytes) *args_bytes = sizeof(agg_args);
    if (rank_info_bytes) *rank_info_bytes = sizeof(agg_rank_info);
    return AGG_OK;
}

const char* agg_last_error(void) { return agg::t_last_error.c_str(); }

int agg_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

// ---------------------------------------------------------------- VMM helpers
int agg_vm_alloc(uint64_t* handle, size_t* allocated_size, size_t size, int device_id) {
    DRV_OR_FAIL();
    if (!handle || !allocated_size) return fail(AGG_EINVAL, "agg_vm_alloc: null output");
    CUmemAllocationProp ap = phys_prop(device_id);
    size_t g = 0;
    AGG_DRV(D.cuMemGetAllocationGranularity(&g, &ap, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED));
    *allocated_size = round_up(size ? size : 1, g);
    CUmemGenericAllocationHandle h = 0;
    AGG_DRV(D.cuMemCreate(&h, *allocated_size, &ap, 0));
    *handle = static_cast<uint64_t>(h);
    return AGG_OK;
}

int agg_vm_map(uint64_t* ptr, uint64_t handle, size_t size) {
    DRV_OR_FAIL();
    if (!ptr) return fail(AGG_EINVAL, "agg_vm_map: null output");
    CUdeviceptr va = 0;
    AGG_DRV(D.cuMemAddressReserve(&va, size, 0, 0, 0));
    CUresult r = D.cuMemMap(va, size, 0, static_cast<CUmemGenericAllocationHandle>(handle), 0);
    if (r != CUDA_SUCCESS) {
        D.cuMemAddressFree(va, size);
        return check_drv(r, "cuMemMap");
    }
    *ptr = static_cast<uint64_t>(va);
    return AGG_OK;
}

int agg_vm_set_access(uint64_t ptr, size_t size, const int* devices, int ndevices) {
    DRV_OR_FAIL();
    if (!devices || ndevices <= 0) return fail(AGG_EINVAL, "agg_vm_set_access: no devices");
    std::vector<CUmemAccessDesc> ad(ndevices);
    for (int i = 0; i < ndevices; ++i) {
        std::memset(&ad[i], 0, sizeof(ad[i]));
        ad[i].location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        ad[i].location.id = devices[i];
        ad[i].flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    }
    AGG_DRV(D.cuMemSetAccess(static_cast<CUdeviceptr>(ptr), size, ad.data(), ndevices));
    return AGG_OK;
}

int agg_vm_unmap_free(uint64_t ptr, size_t size) {
    DRV_OR_FAIL();
    AGG_DRV(D.cuMemUnmap(static_cast<CUdeviceptr>(ptr), size));
    AGG_DRV(D.cuMemAddressFree(static_cast<CUdeviceptr>(ptr), size));
    return AGG_OK;
}

int agg_vm_release(uint64_t handle) {
    DRV_OR_FAIL();
    AGG_DRV(D.cuMemRelease(static_cast<CUmemGenericAllocationHandle>(handle)));
    return AGG_OK;
}

// ---------------------------------------------------------------- in-process init
int agg_spmm_init(int rank, int world, int device, size_t data_bytes, agg_rank_info* out) {
    if (rank < 0 || rank >= AGG_MAX_RANKS || world < 1 || world > AGG_MAX_RANKS || rank >= world)
        return fail(AGG_EINVAL, "agg_spmm_init: rank %d / world %d", rank, world);
    if (device != rank)
        // The multicast object is created over devices 0..world-1 (vmm/multimem.cu:77-85):
        // a remapped rank->device layout would bind the wrong memory.
        return fail(AGG_EINVAL, "agg_spmm_init: rank %d on device %d is not the identity map", rank, device);
    std::call_once(g_proc.once, [&] {
        g_proc.world = world;
        g_proc.rc = create_mc_all(world, data_bytes);
        g_proc.err = agg::t_last_error;
    });
    if (g_proc.rc != AGG_OK) return fail(g_proc.rc, "multicast setup failed: %s", g_proc.err.c_str());
    if (world != g_proc.world) return fail(AGG_EINVAL, "agg_spmm_init: world %d != %d", world, g_proc.world);
    size_t slab = 0, foff = 0;
    size_t gran = 1;
    slab_geometry(data_bytes, gran, &slab, &foff);
    if (foff > g_proc.flag_off)
        return fail(AGG_EINVAL, "agg_spmm_init: %zu data bytes do not fit the slab created first", data_bytes);

    RankSlot& s = g_slots[rank];
    std::lock_guard<std::mutex> lk(s.mu);
    if (!s.mapped) {
        DRV_OR_FAIL();
        int prev = 0;
        AGG_RT(cudaGetDevice(&prev));
        AGG_RT(cudaSetDevice(device));
        CUmemAllocationProp ap = phys_prop(device);
        CUresult r = D.cuMemCreate(&s.phys, g_proc.slab, &ap, 0);
        if (r != CUDA_SUCCESS) return check_drv(r, "cuMemCreate slab");
        r = D.cuMulticastBindMem(g_proc.mc, 0, s.phys, 0, g_proc.slab, 0);
        if (r != CUDA_SUCCESS) return check_drv(r, "cuMulticastBindMem");
        std::vector<int> all(world);
        for (int i = 0; i < world; ++i) all[i] = i;
        int rc = map_range(&s.uc, g_proc.slab, s.phys, all.data(), world);
        if (rc) return rc;
        rc = map_range(&s.mc, g_proc.slab, g_proc.mc, &device, 1);
        if (rc) return rc;
        rc = zero_flags(s.uc, g_proc.flag_off, device);
        if (rc) return rc;
        cudaSetDevice(prev);
        s.mapped = true;
        g_proc.live.fetch_add(1);
    }
    CUdeviceptr peers[AGG_MAX_RANKS] = {0};
    for (int i = 0; i < world; ++i) peers[i] = g_slots[i].uc;  // 0 until that rank has mapped
    fill_info(out, rank, world, device, s.uc, s.mc, peers, g_proc.slab, g_proc.flag_off);
    return AGG_OK;
}

int agg_spmm_finalize(int rank) {
    if (rank < 0 || rank >= AGG_MAX_RANKS) return fail(AGG_EINVAL, "agg_spmm_finalize: rank %d", rank);
    DRV_OR_FAIL();
    RankSlot& s = g_slots[rank];
    std::lock_guard<std::mutex> lk(s.mu);
    if (!s.mapped) return AGG_OK;
    unmap_range(s.mc, g_proc.slab);
    unmap_range(s.uc, g_proc.slab);
    CUdevice dev;
    if (D.cuDeviceGet(&dev, rank) == CUDA_SUCCESS) D.cuMulticastUnbind(g_proc.mc, dev, 0, g_proc.slab);
    D.cuMemRelease(s.phys);
    s.phys = 0;
    s.uc = 0;
    s.mc = 0;
    s.mapped = false;
    if (g_proc.live.fetch_sub(1) == 1) {
        D.cuMemRelease(g_proc.mc);
        g_proc.mc = 0;
    }
    return AGG_OK;
}

// ---------------------------------------------------------------- multi-process init
int agg_mp_open(int rank, int world, int device, size_t data_bytes, const char* job_id, agg_mp_ctx** out) {
    if (!out || !job_id) return fail(AGG_EINVAL, "agg_mp_open: null argument");
    *out = nullptr;
    if (rank < 0 || world < 1 || world > AGG_MAX_RANKS || rank >= world)
        return fail(AGG_EINVAL, "agg_mp_open: rank %d / world %d", rank, world);
    DRV_OR_FAIL();
    DeviceGuard guard(device);
    if (!guard.ok) return fail(AGG_ECUDA, "agg_mp_open: cannot select device %d", device);
    int rc = check_multicast_supported(device);
    if (rc) return rc;
    agg_mp_ctx* c = new agg_mp_ctx();
    c->rank = rank;
    c->world = world;
    c->device = device;
    c->job = job_id;
    for (int i = 0; i < AGG_MAX_RANKS; ++i) {
        c->phys_fd[i] = -1;
        c->peer_phys[i] = 0;
        c->peer_uc[i] = 0;
    }
    size_t gran = 0;
    rc = multicast_granularity(world, 512ull << 20, &gran);
    if (rc) {
        delete c;
        return rc;
    }
    slab_geometry(data_bytes, gran, &c->slab, &c->flag_off);

    // physical slab of this GPU, exportable
    CUmemAllocationProp ap = phys_prop(device);
    CUresult r = D.cuMemCreate(&c->phys, c->slab, &ap, 0);
    if (r != CUDA_SUCCESS) {
        delete c;
        return check_drv(r, "cuMemCreate slab");
    }
    r = D.cuMemExportToShareableHandle(&c->phys_fd[rank], c->phys, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
    if (r != CUDA_SUCCESS) {
        agg_mp_close(c);
        return check_drv(r, "cuMemExportToShareableHandle slab");
    }
    if (rank == 0) {
        CUmulticastObjectProp mp;
        std::memset(&mp, 0, sizeof(mp));
        mp.numDevices = static_cast<unsigned>(world);
        mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
        mp.size = c->slab;
        r = D.cuMulticastCreate(&c->mc, &mp);
        if (r != CUDA_SUCCESS) {
            agg_mp_close(c);
            return check_drv(r, "cuMulticastCreate");
        }
        r = D.cuMemExportToShareableHandle(&c->mc_fd, c->mc, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
        if (r != CUDA_SUCCESS) {
            agg_mp_close(c);
            return check_drv(r, "cuMemExportToShareableHandle multicast");
        }
    }
    // listening socket for the peers' handles
    if (world > 1) {
        int s = socket(AF_UNIX, SOCK_STREAM, 0);
        if (s < 0) {
            agg_mp_close(c);
            return fail(AGG_ESYS, "socket: %s", strerror(errno));
        }
        sockaddr_un a;
        socklen_t len = 0;
        rc = make_addr(sock_name(c->job, rank), &a, &len);
        if (rc || bind(s, reinterpret_cast<sockaddr*>(&a), len) != 0 || listen(s, 2 * AGG_MAX_RANKS) != 0) {
            int e = errno;
            close(s);
            agg_mp_close(c);
            return rc ? rc : fail(AGG_ESYS, "bind/listen: %s", strerror(e));
        }
        c->listen_fd = s;
    }
    *out = c;
    return AGG_OK;
}

int agg_mp_exchange(agg_mp_ctx* c) {
    if (!c) return fail(AGG_EINVAL, "agg_mp_exchange: null ctx");
    if (c->exchanged) return AGG_OK;
    if (c->world == 1) {
        c->exchanged = true;
        return AGG_OK;
    }
    // send: own slab fd to everybody; rank 0 adds the multicast fd
    for (int p = 0; p < c->world; ++p) {
        if (p == c->rank) continue;
        int fds[2] = {c->phys_fd[c->rank], c->mc_fd};
        int rc = send_fds(sock_name(c->job, p), c->rank, fds, c->rank == 0 ? 2 : 1);
        if (rc) return rc;
    }
    // receive one message from every peer
    for (int i = 0; i < c->world - 1; ++i) {
        int from = -1, n = 0, fds[4] = {-1, -1, -1, -1};
        int rc = recv_fds(c->listen_fd, &from, fds, &n);
        if (rc) return rc;
        if (from < 0 || from >= c->world || from == c->rank || n < 1)
            return fail(AGG_ESYS, "bad handle message from rank %d", from);
        c->phys_fd[from] = fds[0];
        if (from == 0) {
            if (n != 2) return fail(AGG_ESYS, "rank 0 sent no multicast handle");
            c->mc_fd = fds[1];
        }
    }
    close(c->listen_fd);
    c->listen_fd = -1;
    c->exchanged = true;
    return AGG_OK;
}

int agg_mp_add_device(agg_mp_ctx* c) {
    if (!c || !c->exchanged) return fail(AGG_ESTATE, "agg_mp_add_device: exchange first");
    if (c->added) return AGG_OK;
    DRV_OR_FAIL();
    DeviceGuard guard(c->device);
    if (c->rank != 0) {
        AGG_DRV(D.cuMemImportFromShareableHandle(&c->mc, reinterpret_cast<void*>(static_cast<uintptr_t>(c->mc_fd)),
                                                  CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR));
    }
    CUdevice dev;
    AGG_DRV(D.cuDeviceGet(&dev, c->device));
    AGG_DRV(D.cuMulticastAddDevice(c->mc, dev));
    c->added = true;
    return AGG_OK;
}

int agg_mp_bind(agg_mp_ctx* c, agg_rank_info* out) {
    if (!c || !c->added) return fail(AGG_ESTATE, "agg_mp_bind: add_device and a barrier first");
    DRV_OR_FAIL();
    if (!c->bound) {
        DeviceGuard guard(c->device);
        AGG_DRV(D.cuMulticastBindMem(c->mc, 0, c->phys, 0, c->slab, 0));
        int rc = map_range(&c->uc, c->slab, c->phys, &c->device, 1);
        if (rc) return rc;
        rc = map_range(&c->mcva, c->slab, c->mc, &c->device, 1);
        if (rc) return rc;
        for (int p = 0; p < c->world; ++p) {
            if (p == c->rank) {
                c->peer_uc[p] = c->uc;
                continue;
            }
            AGG_DRV(D.cuMemImportFromShareableHandle(&c->peer_phys[p],
                                                      reinterpret_cast<void*>(static_cast<uintptr_t>(c->phys_fd[p])),
                                                      CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR));
            rc = map_range(&c->peer_uc[p], c->slab, c->peer_phys[p], &c->device, 1);
            if (rc) return rc;
        }
        rc = zero_flags(c->uc, c->flag_off, c->device);
        if (rc) return rc;
        c->bound = true;
    }
    fill_info(out, c->rank, c->world, c->device, c->uc, c->mcva, c->peer_uc, c->slab, c->flag_off);
    return AGG_OK;
}

int agg_mp_close(agg_mp_ctx* c) {
    if (!c) return AGG_OK;
    const DriverApi& D = driver();
    if (D.ok) {
        DeviceGuard guard(c->device);
        cudaDeviceSynchronize();  // nothing of ours may still touch the mappings
        for (int p = 0; p < c->world && p < AGG_MAX_RANKS; ++p) {
            if (p != c->rank && c->peer_uc[p]) unmap_range(c->peer_uc[p], c->slab);
            if (c->peer_phys[p]) D.cuMemRelease(c->peer_phys[p]);
        }
        if (c->mcva) unmap_range(c->mcva, c->slab);
        if (c->uc) unmap_range(c->uc, c->slab);
        if (c->bound) {
            CUdevice dev;
            if (D.cuDeviceGet(&dev, c->device) == CUDA_SUCCESS) D.cuMulticastUnbind(c->mc, dev, 0, c->slab);
        }
        if (c->phys) D.cuMemRelease(c->phys);
        if (c->mc) D.cuMemRelease(c->mc);
    }
    for (int p = 0; p < AGG_MAX_RANKS; ++p)
        if (c->phys_fd[p] >= 0) close(c->phys_fd[p]);
    if (c->mc_fd >= 0) close(c->mc_fd);
    if (c->listen_fd >= 0) close(c->listen_fd);
    delete c;
    return AGG_OK;
}

}  // extern "C"
