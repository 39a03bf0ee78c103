// multi_gpu.cpp -- the reference's multi-GPU C ABI (csrc/cuda/multi_gpu.cu:37-160,
// declared in csrc/core/wisp_engine.h:656-665): a single-process NCCL pipeline
// over n GPUs and 2-GPU peer copies, with the same signatures and return codes
// (0 = ok, -1 = failure).
//
// NCCL is loaded at first use with dlopen("libnccl.so.2"): inside a process that
// already loaded NCCL (torch) the same library is reused, and without NCCL the
// pipeline calls fail with -1 and wisp_nccl_available() returns 0 -- the
// reference's WISP_HAS_NCCL=OFF build (multi_gpu.cu:135-160).
//
// Semantics kept from the reference: wisp_pipeline_init builds one communicator
// per GPU with ncclCommInitAll (stage i = gpu_indices[i]); send/recv move n fp32
// values between the stage of the *current device* and `peer_stage` on stream
// `s`.  As with any single-process multi-GPU NCCL use, a matching send and
// receive must be issued from different host threads (or the peer's call must
// not wait for this one); the multi-process layer pipeline of this build
// (wisp_b200/pipeline.py, torch.distributed) is the path the benchmarks use.

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <vector>

namespace {

struct Nccl {
    void* h = nullptr;
    ncclResult_t (*comm_init_all)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t,
                         cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    bool ok = false;
};

Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        n.h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!n.h) return;
        n.comm_init_all =
            reinterpret_cast<decltype(n.comm_init_all)>(dlsym(n.h, "ncclCommInitAll"));
        n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(n.h, "ncclCommDestroy"));
        n.send = reinterpret_cast<decltype(n.send)>(dlsym(n.h, "ncclSend"));
        n.recv = reinterpret_cast<decltype(n.recv)>(dlsym(n.h, "ncclRecv"));
        n.ok = n.comm_init_all && n.comm_destroy && n.send && n.recv;
    });
    return n;
}

struct Pipeline {
    std::mutex mu;
    std::vector<int> devs;
    std::vector<ncclComm_t> comms;
};

Pipeline& pipe() {
    static Pipeline p;
    return p;
}

// stage of the current device, or -1
int my_stage(const Pipeline& p) {
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess) return -1;
    for (size_t i = 0; i < p.devs.size(); ++i)
        if (p.devs[i] == d) return (int)i;
    return -1;
}

// The current device's communicator, if the pipeline holds it and peer_stage exists.
bool comm_for(int peer_stage, ncclComm_t* out) {
    if (!nccl().ok) return false;
    Pipeline& p = pipe();
    std::lock_guard<std::mutex> g(p.mu);
    const int me = my_stage(p);
    if (me < 0 || peer_stage < 0 || peer_stage >= (int)p.devs.size()) return false;
    *out = p.comms[(size_t)me];
    return true;
}

}  // namespace

extern "C" int wisp_nccl_available(void) { return nccl().ok ? 1 : 0; }

extern "C" int wisp_pipeline_init(const int* gpu_indices, int n) {
    Nccl& N = nccl();
    if (!N.ok || !gpu_indices || n <= 0) return -1;
    Pipeline& p = pipe();
    std::lock_guard<std::mutex> g(p.mu);
    if (!p.comms.empty()) return -1;  // already initialised: shut down first
    std::vector<ncclComm_t> comms((size_t)n, nullptr);
    // NCCL selects each communicator's device while it builds them: the caller's
    // current device is restored afterwards
    int cur = 0;
    cudaGetDevice(&cur);
    const ncclResult_t r = N.comm_init_all(comms.data(), n, gpu_indices);
    cudaSetDevice(cur);
    if (r != ncclSuccess) return -1;
    p.devs.assign(gpu_indices, gpu_indices + n);
    p.comms = comms;
    return 0;
}

extern "C" void wisp_pipeline_shutdown(void) {
    Nccl& N = nccl();
    Pipeline& p = pipe();
    std::lock_guard<std::mutex> g(p.mu);
    int cur = 0;
    cudaGetDevice(&cur);
    if (N.ok)
        for (ncclComm_t c : p.comms)
            if (c) N.comm_destroy(c);
    cudaSetDevice(cur);  // as in init: the caller's current device is kept
    p.comms.clear();
    p.devs.clear();
}

extern "C" int wisp_pipeline_send_activation(const float* x, int n, int peer_stage,
                                             cudaStream_t s) {
    Nccl& N = nccl();
    ncclComm_t c = nullptr;
    if (!comm_for(peer_stage, &c) || !x || n < 0) return -1;
    // not under the lock: the peer thread's matching receive must be able to enter
    return N.send(x, (size_t)n, ncclFloat32, peer_stage, c, s) == ncclSuccess ? 0 : -1;
}

extern "C" int wisp_pipeline_recv_activation(float* x, int n, int peer_stage, cudaStream_t s) {
    Nccl& N = nccl();
    ncclComm_t c = nullptr;
    if (!comm_for(peer_stage, &c) || !x || n < 0) return -1;
    return N.recv(x, (size_t)n, ncclFloat32, peer_stage, c, s) == ncclSuccess ? 0 : -1;
}

// 2-GPU peer access both ways (multi_gpu.cu:37-56); already-enabled counts as ok.
extern "C" int wisp_peer_enable(int dev_a, int dev_b) {
    int ab = 0, ba = 0;
    if (cudaDeviceCanAccessPeer(&ab, dev_a, dev_b) != cudaSuccess ||
        cudaDeviceCanAccessPeer(&ba, dev_b, dev_a) != cudaSuccess || !ab || !ba)
        return -1;
    int cur = 0;
    cudaGetDevice(&cur);
    int rc = 0;
    for (int k = 0; k < 2 && rc == 0; ++k) {
        const int from = k ? dev_b : dev_a, to = k ? dev_a : dev_b;
        cudaSetDevice(from);
        const cudaError_t e = cudaDeviceEnablePeerAccess(to, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled)
            cudaGetLastError();  // clear the sticky-free error state
        else if (e != cudaSuccess)
            rc = -1;
    }
    cudaSetDevice(cur);
    return rc;
}

// Peer copy on stream s (multi_gpu.cu:58-65).
extern "C" int wisp_peer_copy_async(void* dst, int dst_dev, const void* src, int src_dev,
                                    size_t n, cudaStream_t s) {
    if (!dst || !src) return -1;
    return cudaMemcpyPeerAsync(dst, dst_dev, src, src_dev, n, s) == cudaSuccess ? 0 : -1;
}
