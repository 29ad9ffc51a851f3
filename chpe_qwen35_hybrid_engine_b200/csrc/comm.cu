// comm.cu -- the tensor-parallel exchanges over NVLink peer memory (72B
// shape): after the O and down projections every rank holds an fp32 partial
// [M][H] of the block output and the hidden state needs hidden += the sum of
// the ranks' partials; after the vocabulary-split LM head every rank holds
// the argmax of its shard and needs the global one.
//
// Each rank owns, in its own memory, a receive area of 2 x world tagged slots
// of Mmax x H 8-byte words, mapped into every peer with CUDA IPC.  A word is
// one value and the epoch of the exchange it belongs to (value bits |
// epoch << 32), written by the sending rank with one 64-bit store -- single-
// copy atomic, so a receiver that reads the word sees the value and its epoch
// together.  An exchange is then one NVLink trip: every rank
//   1. reads the epoch (a per-rank counter advanced at the end of every
//      exchange; every rank runs the same sequence of exchanges, so epochs
//      agree),
//   2. stores its values into slot [epoch & 1][rank] of every peer (plain P2P
//      stores; no TMA, no multicast, no flags, no fences),
//   3. polls its own slots [epoch & 1][r] until each word carries the epoch
//      -- bounded by 1 s of %globaltimer for all of a thread's words, after
//      which it records an error,
//   4. combines in rank order (its own values read locally), so every rank
//      computes the same bits.
// Slots alternate with the epoch's parity: a rank writes a slot again two
// epochs later only, after the exchange in between, which needed every
// peer's values -- sent by that peer after its previous kernel, the one that
// read the slot, had finished (stream order; each kernel waits for its
// predecessor before it starts).
//
// A wait that expires leaves the ranks' epochs out of step.  So a thread whose
// wait expires marks the comm object failed -- in its device memory and in a
// mapped host word -- and the epoch stops advancing; every later exchange on a
// failed object returns at once with an error, on the host (the entry points
// refuse) and on the device (a launch already queued, e.g. in a CUDA graph,
// skips the exchange and records the error).  chpe_comm_reset, called on
// every rank between two host barriers, clears the epochs, the slots (their
// epochs restart at 1) and the mark.
//
// The all-reduce also runs fused into the RMSNorm fill that consumes the
// hidden state (prep.cu, chpe_allreduce_fill_dev), with the same slots.
#include <cstring>

#include "../../include/chpe_b200.h"
#include "common.cuh"
#include "internal.h"

namespace chpe {
namespace {

constexpr int kCommThreads = 256;
constexpr int kCommChunk = 1024;  // values per CTA (4 per thread)
static_assert(kCommMaxRanksDev == kCommMaxRanks, "one rank limit");

__device__ __forceinline__ void mark_failed(unsigned *ctr, volatile unsigned *host_failed, int *err) {
    atomicExch(err, kErrCommWait);
    atomicExch(&ctr[2], 1u);  // failed: no later exchange on this object until a reset
    *host_failed = 1u;
}

// The last CTA of a launch advances the epoch for the next exchange (not
// after a failure: the object then stays failed until chpe_comm_reset).
__device__ __forceinline__ void advance_epoch(unsigned *ctr, unsigned epoch, unsigned ctas) {
    __threadfence();
    if (atomicAdd(&ctr[1], 1u) == ctas - 1) {
        ctr[1] = 0u;
        if (!atomicAdd(&ctr[2], 0u)) ctr[0] = epoch;
    }
}

__global__ void __launch_bounds__(kCommThreads) chpe_allreduce_residual_kernel(const CommPeers peers, int world, int rank,
                                                                          size_t slot_elems,
                                                                          const float *__restrict__ part,
                                                                          float *__restrict__ hidden, int n,
                                                                          unsigned *__restrict__ ctr,
                                                                          volatile unsigned *host_failed,
                                                                          int *__restrict__ err) {
    pdl_begin();  // the partial is the previous kernel's output
    // ctr[0] epoch, ctr[1] arrival ticket, ctr[2] failed mark
    if (*reinterpret_cast<volatile unsigned *>(&ctr[2])) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(err, kErrCommFailed);
        return;
    }
    const unsigned epoch = *reinterpret_cast<volatile unsigned *>(&ctr[0]) + 1u;
    const int i0 = blockIdx.x * kCommChunk;
    const size_t slot = ((size_t)(epoch & 1u) * world + rank) * slot_elems;
    float v[kCommChunk / kCommThreads];
#pragma unroll
    for (int j = 0; j < kCommChunk / kCommThreads; ++j) {
        const int i = i0 + threadIdx.x + j * kCommThreads;
        v[j] = i < n ? part[i] : 0.0f;
        if (i < n)
            for (int r = 0; r < world; ++r)
                if (r != rank) st_tagged(peers.tagged[r] + slot + i, v[j], epoch);
    }
    const unsigned long long *own = peers.tagged[rank] + (size_t)(epoch & 1u) * world * slot_elems;
    const unsigned long long t0 = global_timer_ns();
    bool ok = true;
    constexpr int NV = kCommChunk / kCommThreads;
    size_t idx[NV];
    bool valid[NV];
    float sums[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        idx[j] = (size_t)(i0 + threadIdx.x + j * kCommThreads);
        valid[j] = idx[j] < (size_t)n;
    }
    sum_tagged<NV>(own, slot_elems, idx, valid, world, rank, v, epoch, t0, ok, sums);
#pragma unroll
    for (int j = 0; j < NV; ++j)
        if (ok && valid[j]) hidden[idx[j]] += sums[j];
    if (!ok) mark_failed(ctr, host_failed, err);
    __syncthreads();
    if (threadIdx.x == 0) advance_epoch(ctr, epoch, gridDim.x);
}

// The vocabulary-split LM head's argmax: every rank holds, for each of M
// rows, the (max value, index) of its shard; afterwards every rank holds the
// global pair -- the largest value, ties to the smaller global index, as
// src/engine.zig:1098-1110 computeArgmax breaks them within one shard.  One
// CTA: thread m < M sends row m's value and global index as two tagged words,
// waits for every peer's pair and merges the pairs in rank order.
__global__ void __launch_bounds__(32) chpe_argmax_merge_kernel(const CommPeers peers, int world, int rank,
                                                               size_t slot_elems, int *__restrict__ idx,
                                                               float *__restrict__ maxv, int M, int index_base,
                                                               unsigned *__restrict__ ctr,
                                                               volatile unsigned *host_failed,
                                                               int *__restrict__ err) {
    pdl_begin();  // the local argmax is the previous kernel's output
    if (*reinterpret_cast<volatile unsigned *>(&ctr[2])) {
        if (threadIdx.x == 0) atomicExch(err, kErrCommFailed);
        return;
    }
    const unsigned epoch = *reinterpret_cast<volatile unsigned *>(&ctr[0]) + 1u;
    const int m = threadIdx.x;
    bool ok = true;
    if (m < M) {
        const float v = maxv[m];
        const int gi = idx[m] + index_base;
        const size_t slot = ((size_t)(epoch & 1u) * world + rank) * slot_elems;
        for (int r = 0; r < world; ++r) {
            if (r == rank) continue;
            st_tagged(peers.tagged[r] + slot + 2 * m, v, epoch);
            st_tagged(peers.tagged[r] + slot + 2 * m + 1, __int_as_float(gi), epoch);
        }
        const unsigned long long *own = peers.tagged[rank] + (size_t)(epoch & 1u) * world * slot_elems;
        const unsigned long long t0 = global_timer_ns();
        float bv = 0.0f;
        int bi = 0;
        unsigned long long wv[kCommMaxRanks], wi[kCommMaxRanks];  // every peer's pair, loaded up front
#pragma unroll
        for (int r = 0; r < kCommMaxRanks; ++r)
            if (r < world && r != rank) {
                wv[r] = ld_tagged(own + (size_t)r * slot_elems + 2 * m);
                wi[r] = ld_tagged(own + (size_t)r * slot_elems + 2 * m + 1);
            }
#pragma unroll
        for (int r = 0; r < kCommMaxRanks; ++r) {
            if (r >= world || !ok) continue;
            float rv = v;
            int ri = gi;
            if (r != rank) {
                rv = settle_tagged(own + (size_t)r * slot_elems + 2 * m, wv[r], epoch, t0, ok);
                ri = __float_as_int(settle_tagged(own + (size_t)r * slot_elems + 2 * m + 1, wi[r], epoch, t0, ok));
            }
            if (r == 0 || rv > bv || (rv == bv && ri < bi)) {
                bv = rv;
                bi = ri;
            }
        }
        if (ok) {
            idx[m] = bi;
            maxv[m] = bv;
        }
    }
    if (!ok) mark_failed(ctr, host_failed, err);
    __syncthreads();
    if (m == 0) advance_epoch(ctr, epoch, 1);
}

}  // namespace
}  // namespace chpe

using namespace chpe;

static size_t recv_bytes(int world, size_t max_elems) {
    return 2 * (size_t)world * max_elems * sizeof(unsigned long long);
}

struct chpe_comm {
    chpe_ctx *ctx = nullptr;
    int world = 0, rank = 0;
    size_t max_elems = 0;                // Mmax * H, rounded up to whole chunks
    unsigned long long *recv = nullptr;  // own receive area [2][world][max_elems] tagged words
    unsigned *epoch = nullptr;           // own epoch counter, arrival ticket and failed mark
    unsigned *host_failed = nullptr;     // mapped pinned host word: set by a kernel whose wait expired
    unsigned *host_failed_dev = nullptr;
    CommPeers peers;
    bool opened[kCommMaxRanks] = {false};
    cudaIpcMemHandle_t handle_recv;
};

int *chpe_ctx_error_word(chpe_ctx *ctx);

extern "C" int chpe_comm_create(chpe_ctx *ctx, int world, int rank, size_t max_elems, chpe_comm **out) {
    if (!ctx || !out) return CHPE_EINVAL;
    *out = nullptr;
    if (world < 1 || world > kCommMaxRanks || rank < 0 || rank >= world || max_elems < 1) return CHPE_EINVAL;
    chpe_comm *c = new chpe_comm();
    c->ctx = ctx;
    c->world = world;
    c->rank = rank;
    c->max_elems = (max_elems + kCommChunk - 1) / kCommChunk * kCommChunk;
    memset(&c->peers, 0, sizeof c->peers);
    cudaError_t e = cudaMalloc(&c->recv, recv_bytes(world, c->max_elems));
    if (e == cudaSuccess) e = cudaMalloc(&c->epoch, 256);
    if (e == cudaSuccess) e = cudaMemset(c->recv, 0, recv_bytes(world, c->max_elems));  // epoch 0: no exchange yet
    if (e == cudaSuccess) e = cudaMemset(c->epoch, 0, 256);
    if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void **>(&c->host_failed), sizeof(unsigned),
                                            cudaHostAllocMapped);
    if (e == cudaSuccess) {
        *c->host_failed = 0u;
        e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&c->host_failed_dev), c->host_failed, 0);
    }
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&c->handle_recv, c->recv);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(c->recv);
        cudaFree(c->epoch);
        if (c->host_failed) cudaFreeHost(c->host_failed);
        delete c;
        cudaGetLastError();
        return CHPE_ECUDA;
    }
    c->peers.tagged[rank] = c->recv;
    *out = c;
    return CHPE_OK;
}

extern "C" size_t chpe_comm_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int chpe_comm_handle(const chpe_comm *c, void *out) {
    if (!c || !out) return CHPE_EINVAL;
    memcpy(out, &c->handle_recv, sizeof(cudaIpcMemHandle_t));
    return CHPE_OK;
}

extern "C" int chpe_comm_open_peers(chpe_comm *c, const void *handles) {
    if (!c || !handles) return CHPE_EINVAL;
    const size_t hb = chpe_comm_handle_bytes();
    for (int r = 0; r < c->world; ++r) {
        if (r == c->rank || c->opened[r]) continue;
        cudaIpcMemHandle_t hr;
        memcpy(&hr, static_cast<const uint8_t *>(handles) + r * hb, sizeof hr);
        void *pr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&pr, hr, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return CHPE_ECUDA;
        }
        c->peers.tagged[r] = static_cast<unsigned long long *>(pr);
        c->opened[r] = true;
    }
    return CHPE_OK;
}

static bool peers_open(const chpe_comm *c) {
    for (int r = 0; r < c->world; ++r)
        if (!c->peers.tagged[r]) return false;
    return true;
}

extern "C" int chpe_allreduce_residual_dev(chpe_comm *c, const float *part, float *hidden, size_t n, void *stream) {
    if (!c || !part || !hidden) return CHPE_EINVAL;
    if (n > c->max_elems) return CHPE_EINVAL;
    if (!peers_open(c)) return CHPE_ENOENT;
    // a failed object (a bounded wait expired) takes no exchange until chpe_comm_reset
    if (*reinterpret_cast<volatile unsigned *>(c->host_failed)) return CHPE_ETIMEOUT;
    if (n == 0) return CHPE_OK;
    const unsigned chunks = (unsigned)((n + kCommChunk - 1) / kCommChunk);
    cudaError_t e = launch_pdl(chpe_allreduce_residual_kernel, dim3(chunks), dim3(kCommThreads), 0,
                               static_cast<cudaStream_t>(stream), c->peers, c->world, c->rank, c->max_elems, part,
                               hidden, (int)n, c->epoch, c->host_failed_dev, chpe_ctx_error_word(c->ctx));
    return e == cudaSuccess ? CHPE_OK : CHPE_ECUDA;
}

extern "C" int chpe_argmax_merge_dev(chpe_comm *c, int *idx, float *maxv, int M, int index_base, void *stream) {
    if (!c || !idx || !maxv) return CHPE_EINVAL;
    if (M < 1 || M > 32 || (size_t)2 * M > c->max_elems) return CHPE_EINVAL;
    if (!peers_open(c)) return CHPE_ENOENT;
    if (*reinterpret_cast<volatile unsigned *>(c->host_failed)) return CHPE_ETIMEOUT;
    cudaError_t e = launch_pdl(chpe_argmax_merge_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
                               c->peers, c->world, c->rank, c->max_elems, idx, maxv, M, index_base, c->epoch,
                               c->host_failed_dev, chpe_ctx_error_word(c->ctx));
    return e == cudaSuccess ? CHPE_OK : CHPE_ECUDA;
}

// The exchange state a fused fill needs (launch_xfill_f16): refuses like
// chpe_allreduce_residual_dev, and with CHPE_ENOTSUP when n partials do not
// fit the receive area.
int comm_fill_exchange(chpe_comm *c, const float *part, float *hidden, size_t n, FillExchange *out) {
    if (!c || !part || !hidden || !out) return CHPE_EINVAL;
    if (n > c->max_elems) return CHPE_ENOTSUP;
    if (!peers_open(c)) return CHPE_ENOENT;
    if (*reinterpret_cast<volatile unsigned *>(c->host_failed)) return CHPE_ETIMEOUT;
    FillExchange ex;
    ex.peers = c->peers;
    ex.world = c->world;
    ex.rank = c->rank;
    ex.slot_elems = c->max_elems;
    ex.part = part;
    ex.hidden = hidden;
    ex.ctr = c->epoch;
    ex.host_failed = c->host_failed_dev;
    ex.err = chpe_ctx_error_word(c->ctx);
    *out = ex;
    return CHPE_OK;
}

chpe_ctx *comm_ctx(const chpe_comm *c) { return c ? c->ctx : nullptr; }

extern "C" int chpe_comm_failed(const chpe_comm *c) {
    if (!c) return CHPE_EINVAL;
    return *reinterpret_cast<volatile unsigned *>(c->host_failed) ? 1 : 0;
}

extern "C" int chpe_comm_reset(chpe_comm *c) {
    if (!c) return CHPE_EINVAL;
    // every kernel of this process that may touch the object has finished
    cudaError_t e = cudaDeviceSynchronize();
    // the slots carry old epochs, which restart at 1 after the reset
    if (e == cudaSuccess) e = cudaMemset(c->recv, 0, recv_bytes(c->world, c->max_elems));
    if (e == cudaSuccess) e = cudaMemset(c->epoch, 0, 256);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaGetLastError();
        return CHPE_ECUDA;
    }
    *reinterpret_cast<volatile unsigned *>(c->host_failed) = 0u;
    return CHPE_OK;
}

extern "C" int chpe_comm_destroy(chpe_comm *c) {
    if (!c) return CHPE_EINVAL;
    cudaDeviceSynchronize();
    for (int r = 0; r < c->world; ++r)
        if (c->opened[r]) cudaIpcCloseMemHandle(c->peers.tagged[r]);
    cudaFree(c->recv);
    cudaFree(c->epoch);
    cudaFreeHost(c->host_failed);
    delete c;
    return CHPE_OK;
}
