// Step-level exchange between the ranks of a peer group over NVLink: one
// float's max across the ranks (the whole tensor's amax before a per-tensor
// dynamic quantize of row shards) and a barrier (after the GEMM epilogues'
// peer stores). It replaces two one-float NCCL all-reduces per step with one
// tiny kernel each: rank r writes (epoch, value) into slot r of every rank's
// slot array with one 64-bit P2P store, then waits until its own array holds
// the epoch in every slot. Slots live in memory the ranks mapped into each
// other's address space (CUDA IPC), zeroed before the first epoch (1).
//
// Two banks of slots, chosen by the epoch's parity: a rank that has seen
// every word of epoch e may go on and publish epoch e + 1 before a slower
// rank has read its word of epoch e, but it cannot publish e + 2 before that
// rank has published e + 1 (which it does only after reading all of e), so a
// bank is never overwritten while it is still being read.
#include "lcml_device.cuh"
#include "lcml_internal.h"

namespace lcml {
namespace {

constexpr int kMaxPeerRanks = 32;  // one warp: one lane per rank; also the bank stride

__device__ __forceinline__ void st_release_sys_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// One warp. Lane t (t < world) publishes this rank's word to rank t's slot
// array (its own array for t == rank) and then waits for slot t of this
// rank's array to carry `epoch`. The wait is bounded by timeout_ns of the
// global timer; a lane that gives up records kDevTimeoutPeer and the kernel
// returns with *out unchanged.
__global__ void __launch_bounds__(32) k_peer_exchange_max(const float *__restrict__ value, float *__restrict__ out,
                                                          unsigned long long *slots,
                                                          unsigned long long *const *__restrict__ peer_slots,
                                                          int rank, int world, uint32_t epoch,
                                                          unsigned long long timeout_ns, int *err) {
    __threadfence_system();  // the stream's earlier peer stores (the GEMM epilogue's) precede the flag
    const int t = static_cast<int>(threadIdx.x);
    const float v = value ? __ldg(value) : 0.0f;
    const unsigned long long word = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
    const int bank = static_cast<int>(epoch & 1u) * kMaxPeerRanks;
    if (t < world) {
        unsigned long long *dst = (t == rank) ? slots : peer_slots[t < rank ? t : t - 1];
        st_release_sys_u64(dst + bank + rank, word);
    }
    bool ok = true;
    float got = -__int_as_float(0x7f800000);  // -inf: the identity of the max
    if (t < world) {
        const unsigned long long *src = slots + bank + t;
        unsigned long long w = ld_acquire_sys_u64(src);
        if (static_cast<uint32_t>(w >> 32) != epoch) {
            const unsigned long long t0 = global_ns();
            while (static_cast<uint32_t>(w >> 32) != epoch) {
                if (global_ns() - t0 > timeout_ns) {
                    ok = false;
                    break;
                }
                __nanosleep(64);
                w = ld_acquire_sys_u64(src);
            }
        }
        if (ok) got = __uint_as_float(static_cast<uint32_t>(w));
    }
    const bool all_ok = __all_sync(0xffffffffu, ok);
    if (!ok) record_device_error(err, kDevTimeoutPeer);
    // max over the ranks' values: NaN-free by construction (amax ignores NaN)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) got = fmaxf(got, __shfl_xor_sync(0xffffffffu, got, o));
    if (t == 0 && all_ok && out) *out = got;
}

}// namespace
}// namespace lcml

using namespace lcml;

extern "C" int lcml_peer_exchange_max(const float *value, float *out, uint64_t *slots, uint64_t *const *peer_slots,
                                      int rank, int world, uint32_t epoch, uint32_t timeout_us,
                                      lcml_stream_t stream) {
    LCML_CHECK_ARG(world >= 1 && world <= kMaxPeerRanks, "lcml_peer_exchange_max: world %d outside [1, %d]", world,
                   kMaxPeerRanks);
    LCML_CHECK_ARG(rank >= 0 && rank < world, "lcml_peer_exchange_max: rank %d outside [0, %d)", rank, world);
    LCML_CHECK_ARG(epoch != 0, "lcml_peer_exchange_max: epoch 0 is the slots' initial state");
    LCML_CHECK_ARG(slots != nullptr && aligned(slots, 8), "lcml_peer_exchange_max: slots must be 8-byte aligned");
    LCML_CHECK_ARG(world == 1 || peer_slots != nullptr, "lcml_peer_exchange_max: peer_slots is NULL");
    LCML_CHECK_ARG(value == nullptr || out != nullptr, "lcml_peer_exchange_max: value without out");
    LCML_CHECK_ARG(timeout_us > 0, "lcml_peer_exchange_max: timeout_us must be positive");
    k_peer_exchange_max<<<1, 32, 0, to_cuda(stream)>>>(
        value, out, reinterpret_cast<unsigned long long *>(slots),
        reinterpret_cast<unsigned long long *const *>(peer_slots), rank, world, epoch,
        static_cast<unsigned long long>(timeout_us) * 1000ull, device_error_word());
    LCML_LAUNCHED("peer_exchange_max");
    return LCML_OK;
}
