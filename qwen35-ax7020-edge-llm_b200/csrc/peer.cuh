// peer.cuh -- row-sharded launches over the GPUs of one node: where finished
// output rows also go (the other ranks' copies of the full output, mapped
// through CUDA IPC) and the bounded cross-GPU epoch flags that order the
// launches of all ranks.
//
// Protocol: every rank runs the same sequence of launches.  Launch n of a
// rank waits until every rank published epoch n - 1 into this GPU's flag
// array (so the inputs it reads -- rows written by all ranks in launch n - 1
// -- are complete and nobody still reads what it overwrites), and its last
// CTA publishes epoch n into every rank's flag array after all of its rows
// (local and peer stores) are visible system-wide.
#pragma once
#include <cstdint>

namespace qb {

constexpr int kMaxRanks = 8;

struct PeerOut {
    float* y[kMaxRanks];   // the other ranks' full outputs (peer pointers)
    int n;                 // how many
    int row_base;          // global index of this rank's row 0 in a full output row
};

struct SyncArgs {
    const unsigned int* wait_flags;          // this GPU's flags, one per rank
    unsigned int wait_epoch;                 // 0: no wait
    unsigned int* sig_flags[kMaxRanks];      // every rank's flag array (peer pointers)
    unsigned int* sig_ticket;                // zeroed grid ticket of this plan
    unsigned int sig_epoch;                  // 0: no signal
    int world, rank;
    // nullptr: the epochs above are absolute.  Otherwise a nonzero epoch is
    // an offset from the device counter *epoch_base, read when the launch
    // runs (so a captured graph replays fresh epochs once the counter moves)
    const unsigned int* epoch_base;
};

constexpr uint32_t kFlagPolls = 1u << 22;   // bounded wait on peer flags (each poll may sleep)
constexpr uint32_t kErrPeerTimeout = 2u;    // error-word bit of a flag wait that gave up

inline bool sync_args_ok(const SyncArgs& s) {
    return s.world >= 1 && s.world <= kMaxRanks && s.rank >= 0 && s.rank < s.world &&
           (!s.wait_epoch || s.wait_flags) && (!s.sig_epoch || s.sig_ticket);
}

#ifdef __CUDACC__
// Flags are stored and polled relaxed at system scope; the ordering comes
// from fences: the signalling thread's __threadfence_system() before its
// stores (a release pattern), the waiting thread's acq_rel fence after it
// has seen every flag (an acquire pattern).  Measured between two GPUs, a
// round trip costs 4.4 us this way and 5.8 us with release stores and
// acquire polls.
__device__ __forceinline__ unsigned int ld_relaxed_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The epoch a launch uses: e itself, or e + *base (mod 2^32) with a counter.
__device__ __forceinline__ unsigned int epoch_of(unsigned int e, const unsigned int* base) {
    return base ? e + *base : e;
}

// Thread 0 waits until flags[r] >= epoch_of(epoch, base) for every rank r
// (wrap-safe compare), giving up after kFlagPolls polls with kErrPeerTimeout
// in *err; then the whole CTA proceeds.  Every thread of the CTA must call it.
__device__ __forceinline__ void wait_peer_flags(const unsigned int* flags, int world, unsigned int epoch,
                                                const unsigned int* base, unsigned int* err) {
    if (threadIdx.x == 0) {
        epoch = epoch_of(epoch, base);
        for (int r = 0; r < world; r++) {
            uint32_t i = 0;
            while ((int)(ld_relaxed_sys(flags + r) - epoch) < 0) {
                if (++i == kFlagPolls) {
                    if (err) atomicOr(err, kErrPeerTimeout);
                    break;
                }
                __nanosleep(64);
            }
        }
        asm volatile("fence.acq_rel.sys;" ::: "memory");
    }
    __syncthreads();
}

// End of a launch: the last CTA to get here publishes sig_epoch to every
// rank.  Every thread of every CTA must call it after its last store.
__device__ __forceinline__ void signal_peers(const SyncArgs& s) {
    if (!s.sig_epoch) return;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned int t = atomicAdd(s.sig_ticket, 1u);
        if (t == gridDim.x * gridDim.y * gridDim.z - 1) {
            __threadfence_system();
            const unsigned int e = epoch_of(s.sig_epoch, s.epoch_base);
            for (int r = 0; r < s.world; r++) st_relaxed_sys(s.sig_flags[r] + s.rank, e);
            *s.sig_ticket = 0u;   // the plan's next launch is stream-ordered after this one
        }
    }
}
#endif

}  // namespace qb
