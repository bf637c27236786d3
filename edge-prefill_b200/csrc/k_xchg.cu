// k_xchg.cu -- completion wait of the head-parallel output exchange.
//
// In exchange mode every K3 CTA TMA-stores its output tiles into the exchange
// buffer of every rank and then adds to a 64-bit counter there with a
// system-scope release.  This kernel, enqueued on a rank's stream after its
// own K3 call, spins (one thread, acquire loads) until its counter reaches the
// total the host expects from all ranks' calls, so the kernels that follow on
// the stream read complete, visible tiles.  The spin is bounded by
// %globaltimer: on timeout it records kDevWaitExchange and returns.
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

}  // namespace

cudaError_t launch_exchange_wait(const unsigned long long* sig, unsigned long long target, int32_t* err,
                                 uint64_t timeout_ns, cudaStream_t s) {
    k5_exchange_wait<<<1, 32, 0, s>>>(sig, target, err, timeout_ns);
    return cudaGetLastError();
}

}  // namespace epsp
