// agg_main: the reference harness's correctness run (vmm/main.cpp:207-344,
// thread_func2) written against this library's drop-in headers: one process,
// one host thread per GPU, the multicast slab from minfer_spmm_init, inputs from
// fill_random (A shard seed 1000r+1 placed at the start of the rank's slab, B
// seed 1000r+2), one launch_ag_gemm_warp_specialized<128,256,2,5>, and the
// cuBLAS reference_matmul_cublas + check_close of every rank's full output.
// It also checks that A_local_buf received the gathered activation bit-exactly.
//
//   agg_main [world=#GPUs (<=8)] [M=4096] [K=7168] [N=6400]
//
// Exit status 0 when every rank passes.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <barrier>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <thread>
#include <vector>

#include "ag_gemm_warp_specialized.cuh"
#include "multimem.cuh"
#include "random_fill.cuh"
#include "reference_matmul.cuh"

RankState g_rs[8];

namespace {

int g_world = 2;
int g_M = 4096, g_K = 7168, g_N = 6400;
std::unique_ptr<std::barrier<>> g_bar;
std::atomic<bool> g_failed{false};
std::vector<float> g_A_host[8];
std::vector<float> g_B_host[8];

bool ok_cuda(cudaError_t e, const char* what, int rank) {
    if (e == cudaSuccess) return true;
    std::fprintf(stderr, "[rank %d] %s -> %s\n", rank, what, cudaGetErrorString(e));
    return false;
}

// Every rank reaches every barrier, also after a failure, so nobody waits forever.
void sync_point() { g_bar->arrive_and_wait(); }

void rank_main(int r) {
    using fg = ag_gemm_warp_specialized::fused_globals<128, 256, 2>;
    const int M = g_M, K = g_K, N = g_N, M_LOCAL = g_M / g_world;
    bool ok = ok_cuda(cudaSetDevice(r), "cudaSetDevice", r);
    const size_t shard_bytes = static_cast<size_t>(M_LOCAL) * K * sizeof(comm::bf16);
    const size_t data_bytes = ag_gemm_warp_specialized::gather_offset(shard_bytes) +
                              static_cast<size_t>(M) * K * sizeof(comm::bf16);
    if (ok && minfer_spmm_init(r, g_world, r, data_bytes) != 0) {
        std::fprintf(stderr, "[rank %d] SP_MM initialization failed\n", r);
        ok = false;
    }
    if (!ok) g_failed.store(true);
    sync_point();  // every rank's mappings exist
    for (int i = 0; i < g_world; ++i) g_rs[r].peer_addresses[i] = g_rs[i].uc;

    comm::bf16 *B = nullptr, *C = nullptr, *A = nullptr;
    uint32_t* A_ready = nullptr;
    if (!g_failed.load()) {
        ok = ok_cuda(cudaMalloc(&B, sizeof(comm::bf16) * N * K), "malloc B", r) &&
             ok_cuda(cudaMalloc(&C, sizeof(comm::bf16) * M * N), "malloc C", r) &&
             ok_cuda(cudaMalloc(&A, sizeof(comm::bf16) * M * K), "malloc A", r) &&
             ok_cuda(cudaMalloc(&A_ready, sizeof(uint32_t) * 8), "malloc A_ready", r) &&
             ok_cuda(cudaMemset(A_ready, 0, sizeof(uint32_t) * 8), "memset", r);
        if (ok) {
            auto B_view = dist::local_tensor_from_data_ptr<fg::B_local_tensor>(reinterpret_cast<uint64_t>(B), 1, 1, N, K);
            auto A_view = dist::local_tensor_from_data_ptr<fg::A_local_tensor>(g_rs[r].uc, 1, 1, M_LOCAL, K);
            g_B_host[r] = fill_random(B_view, 1000 * r + 2);
            g_A_host[r] = fill_random(A_view, 1000 * r + 1);
            ok = ok_cuda(cudaDeviceSynchronize(), "fill", r);
        }
        if (!ok) g_failed.store(true);
    }
    sync_point();  // every shard is in place

    if (!g_failed.load()) {
        fg g = {
            .A = dist::distributed_tensor_from_data_ptr<fg::A_distributed_tensor>(
                g_rs[r].mc, reinterpret_cast<uint64_t*>(g_rs[r].peer_addresses), 1, 1, M_LOCAL, K),
            .A_local_buf = dist::local_tensor_from_data_ptr<fg::A_local_tensor>(reinterpret_cast<uint64_t>(A), 1, 1, M, K),
            .B = dist::local_tensor_from_data_ptr<fg::B_local_tensor>(reinterpret_cast<uint64_t>(B), 1, 1, N, K),
            .C = dist::local_tensor_from_data_ptr<fg::C_local_tensor>(reinterpret_cast<uint64_t>(C), 1, 1, M, N),
            .A_copy_ready = A_ready,
            .A_copy_epoch = 1,
            .dev_idx = r,
            .M = M,
            .N = N,
        };
        ok = launch_ag_gemm_warp_specialized<128, 256, 2, 5>(g) == 0 &&
             ok_cuda(cudaDeviceSynchronize(), "sync after gemm launch", r);
        if (!ok) g_failed.store(true);
    }
    sync_point();  // every rank's launch is complete before anything is freed

    if (!g_failed.load()) {
        std::vector<float> full_A;
        full_A.reserve(static_cast<size_t>(M) * K);
        for (int s = 0; s < g_world; ++s) full_A.insert(full_A.end(), g_A_host[s].begin(), g_A_host[s].end());
        std::vector<float> gathered = read_back_as_float(A, static_cast<size_t>(M) * K);
        const bool gather_ok = std::memcmp(gathered.data(), full_A.data(), gathered.size() * sizeof(float)) == 0;
        std::vector<float> want = reference_matmul_cublas(full_A, M, K, g_B_host[r], N);
        std::vector<float> got = read_back_as_float(C, static_cast<size_t>(M) * N);
        const bool gemm_ok = check_close(got, want, M, N);
        if (gather_ok && gemm_ok) {
            std::printf("[rank %d] gathered A bit-exact, GEMM correctness check PASS (full %dx%d output)\n", r, M, N);
        } else {
            std::printf("[rank %d] FAILED (gather %s, gemm %s)\n", r, gather_ok ? "ok" : "BAD", gemm_ok ? "ok" : "BAD");
            g_failed.store(true);
        }
    }
    sync_point();
    cudaFree(B);
    cudaFree(C);
    cudaFree(A);
    cudaFree(A_ready);
    sync_point();  // nobody unbinds while another rank may still touch the multicast object
    minfer_spmm_finalize(r);
}

}  // namespace

int main(int argc, char** argv) {
    int devices = 0;
    if (cudaGetDeviceCount(&devices) != cudaSuccess || devices < 1) {
        std::fprintf(stderr, "agg_main: no CUDA device\n");
        return 1;
    }
    g_world = argc > 1 ? std::atoi(argv[1]) : (devices < 8 ? devices : 8);
    if (argc > 2) g_M = std::atoi(argv[2]);
    if (argc > 3) g_K = std::atoi(argv[3]);
    if (argc > 4) g_N = std::atoi(argv[4]);
    if (g_world < 1 || g_world > 8 || g_world > devices || g_M % g_world) {
        std::fprintf(stderr, "agg_main: bad world %d (devices %d) or M %d\n", g_world, devices, g_M);
        return 1;
    }
    std::printf("agg_main: world=%d M=%d K=%d N=%d (per rank %d rows of A)\n", g_world, g_M, g_K, g_N, g_M / g_world);
    g_bar = std::make_unique<std::barrier<>>(g_world);
    std::vector<std::thread> th;
    for (int r = 0; r < g_world; ++r) th.emplace_back(rank_main, r);
    for (auto& t : th) t.join();
    return g_failed.load() ? 1 : 0;
}
