// Classifier-free guidance split across two GPUs (the latency mode of one image): GPU 0 runs
// the unconditional branch, GPU 1 the conditional one, each a single-branch forward, and the
// two noise predictions meet once per step in apply_classifier_free_guidance
// (transformer.cpp:570-602) followed by the scheduler update (scheduler.cpp:272-318).
//
// The exchange and the update are one kernel over NVLink peer memory. Each GPU owns a region
// (the receive buffers and flags of PairLink, kernels.h) that the other maps through CUDA IPC.
// Block i of the kernel
//   1. stores its slice of this GPU's noise prediction into the peer's receive buffer
//      (plain peer stores, 16 bytes per thread), then releases a system-scope increment of
//      the peer's flag i;
//   2. waits (bounded by the handle's wait limit) until its own flag i, incremented by the
//      peer's block i, passes the number of exchanges block i has completed;
//   3. combines the two slices (u + g (c - u)) and applies the scheduler update to the same
//      elements of the latents, which both GPUs hold identically.
// Slices are elementwise, so block i depends on the peer's block i only. The receive buffer is
// double-buffered by exchange parity: the peer's exchange n+2 cannot start before this GPU's
// block i has pushed exchange n+1, which it does only after reading exchange n. The grid is at
// most kPairBlocks blocks, so every block of both grids can be resident at once.
#include <algorithm>

#include "kernels.h"

namespace sana {

namespace {

constexpr int kPairThreads = 256;

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_sys_add(int* p, int v) {
    asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(kPairThreads)
    cfg_pair_kernel(const float* __restrict__ own, PairLink link, int images, int Cl, int HW, long long chunk,
                    float* __restrict__ lat, float* __restrict__ hist_cur, const float* __restrict__ hist_prev,
                    SchedCoef k, int branch, int* err) {
    __shared__ int ready;
    const long long n = static_cast<long long>(images) * Cl * HW;
    const long long lo = blockIdx.x * chunk;
    const long long hi = min(n, lo + chunk);
    const int slot = blockIdx.x;
    const int done = link.count[slot];  // exchanges this slot has completed; only this block writes it
    const long long parity = done & 1;

    float* to_peer = link.peer_recv + parity * link.capacity;
    for (long long e = lo + 4LL * threadIdx.x; e < hi; e += 4LL * blockDim.x)
        *reinterpret_cast<float4*>(to_peer + e) = *reinterpret_cast<const float4*>(own + e);
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        red_release_sys_add(link.peer_flags + slot, 1);
        const uint64_t t0 = global_ns();
        const uint64_t limit = wait_limit_ns(err);
        int ok = 1;
        for (uint32_t it = 0;; ++it) {
            if (ld_acquire_sys(link.flags + slot) > done) break;
            if ((it & 63u) == 0 && global_ns() - t0 > limit) {
                atomicCAS(err, 0, kTimeout);
                ok = 0;
                break;
            }
        }
        if (ok) link.count[slot] = done + 1;
        ready = ok;
    }
    __syncthreads();
    if (!ready) return;

    const float* from_peer = link.recv + parity * link.capacity;
    for (long long e = lo + threadIdx.x; e < hi; e += blockDim.x) {
        // noise is token-major [(b * HW + t) * Cl + c]; latents NCHW [(b * Cl + c) * HW + t]
        const int c = static_cast<int>(e % Cl);
        const long long r = e / Cl;
        const int t = static_cast<int>(r % HW);
        const long long b = r / HW;
        const long long li = (b * Cl + c) * HW + t;
        const float mine = own[e], theirs = from_peer[e];
        const float u = branch == 0 ? mine : theirs;
        const float txt = branch == 0 ? theirs : mine;
        const float guided = u + k.guidance * (txt - u);
        const float x = lat[li];
        const float x0 = x - k.sigma_s * guided;
        const float xn = k.second_order ? k.a * x + k.b * x0 + k.c * (k.inv_r0 * (x0 - hist_prev[li]))
                                        : k.a * x + k.b * x0;
        hist_cur[li] = x0;
        lat[li] = xn;
    }
}

}  // namespace

void cfg_pair_step(const float* own_noise, const PairLink& link, int images, int Cl, int HW, float* lat,
                   float* hist_cur, const float* hist_prev, SchedCoef k, int branch, int* err, cudaStream_t st) {
    const long long n = static_cast<long long>(images) * Cl * HW;
    SANA_REQUIRE(Cl % 4 == 0, "the two-GPU guidance exchange needs latent channels divisible by 4");
    SANA_REQUIRE(n <= link.capacity, "latents exceed the two-GPU exchange buffers");
    SANA_REQUIRE(branch == 0 || branch == 1, "branch must be 0 (unconditional) or 1 (conditional)");
    const long long blocks = std::min<long long>(kPairBlocks, (n + 2047) / 2048);
    const long long chunk = ((n + blocks - 1) / blocks + 3) / 4 * 4;
    const int grid = static_cast<int>((n + chunk - 1) / chunk);
    cfg_pair_kernel<<<grid, kPairThreads, 0, st>>>(own_noise, link, images, Cl, HW, chunk, lat, hist_cur, hist_prev, k,
                                                   branch, err);
    SANA_CUDA(cudaGetLastError());
}

}  // namespace sana
