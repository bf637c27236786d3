// k_xchg.cu -- completion signal and wait of the head-parallel output exchange.
//
// In exchange mode every K3 CTA stores its output tiles into the exchange
// buffer of every rank (coalesced thread stores over NVLink) and exits.
// The signal kernel, enqueued right after K3 on the same stream, starts only
// when the K3 grid has completed -- with all of its stores performed -- and
// adds the number of (token, query head) rows that call covered to a 64-bit
// counter on every rank with a system-scope release.  The wait kernel,
// enqueued before the kernels that read a slot, spins (one thread, acquire
// loads) until its counter reaches the total the host expects from all
// ranks' calls.  The spin is bounded by %globaltimer: on timeout it records
// kDevWaitExchange and returns.
#include <cuda_runtime.h>

#include "epsp_kernels.h"
#include "tc100.cuh"

namespace epsp {
namespace {

__global__ void k5_exchange_wait(const unsigned long long* sig, unsigned long long target, int32_t* err,
                                 uint64_t timeout_ns) {
    if (threadIdx.x != 0) return;
    const uint64_t t0 = tc::globaltimer_ns();
    for (;;) {
        if (tc::ld_acquire_sys(sig) >= target) break;
        if (tc::globaltimer_ns() - t0 > timeout_ns) {
            atomicCAS(err, 0, kDevWaitExchange);
            break;
        }
        __nanosleep(128);
    }
}

struct SigList {
    unsigned long long* p[kMaxDest];
};

__global__ void k5_exchange_signal(const SigList sig, int n, unsigned long long value) {
    if ((int)threadIdx.x < n) {
        __threadfence_system();
        tc::red_add_release_sys(sig.p[threadIdx.x], value);
    }
}

}  // namespace

cudaError_t launch_exchange_signal(unsigned long long* const* sig, int n, unsigned long long value, cudaStream_t s) {
    if (n < 1 || n > kMaxDest) return cudaErrorInvalidValue;
    SigList l{};
    for (int i = 0; i < n; ++i) l.p[i] = sig[i];
    k5_exchange_signal<<<1, 32, 0, s>>>(l, n, value);
    return cudaGetLastError();
}

cudaError_t launch_exchange_wait(const unsigned long long* sig, unsigned long long target, int32_t* err,
                                 uint64_t timeout_ns, cudaStream_t s) {
    k5_exchange_wait<<<1, 32, 0, s>>>(sig, target, err, timeout_ns);
    return cudaGetLastError();
}

}  // namespace epsp
