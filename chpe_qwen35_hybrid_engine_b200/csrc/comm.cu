// comm.cu -- one-shot all-reduce over NVLink peer memory for tensor
// parallelism (72B shape): after the O and down projections every rank holds
// an fp32 partial [M][H] of the block output; the hidden state needs
// hidden += sum over ranks of the partials.
//
// Each rank owns, in its own memory, a receive area of 2 x world slots of
// Mmax x H floats plus arrival flags [world][chunks], mapped into every peer
// with CUDA IPC.  One kernel per all-reduce, one CTA per chunk of 1024 floats
// (M = 1, H = 8192: 8 CTAs); CTA c, independently of the others:
//   1. reads the epoch (a per-rank counter advanced at the end of every
//      all-reduce; every rank runs the same sequence, so epochs agree),
//   2. stores chunk c of this rank's partial into slot [epoch & 1][rank] of
//      every peer's receive area (P2P stores over NVLink; no TMA, no
//      multicast), then one thread per peer raises flag [rank][c] there with a
//      system-scope release store,
//   3. waits until flag [r][c] of its own area reaches the epoch for every
//      peer r -- bounded by 1 s of %globaltimer, after which it records an
//      error and returns,
//   4. hidden[i] += partial_0[i] + partial_1[i] + ... in rank order (its own
//      partial read locally), so every rank computes the same bits.
// Slots alternate with the epoch's parity: a rank can only rewrite a chunk's
// slot two epochs later, after it has seen every peer's flag for that chunk in
// the epoch in between, which each peer raises only after it finished reading
// the older slot.
//
// A wait that expires leaves the ranks' epochs out of step, and a later
// exchange could pair slots of different epochs without noticing.  So a CTA
// whose wait expires marks the comm object failed -- in its device memory and
// in a mapped host word -- and the epoch stops advancing; every later
// all-reduce on a failed object returns at once with an error, on the host
// (chpe_allreduce_residual_dev refuses) and on the device (a launch already
// queued, e.g. in a CUDA graph, skips the exchange and records the error).
// chpe_comm_reset, called on every rank between two host barriers, clears the
// epochs, the flags and the mark.
#include <cstring>

#include "../../include/chpe_b200.h"
#include "common.cuh"
#include "internal.h"

namespace chpe {
namespace {

constexpr int kCommThreads = 256;
constexpr int kCommChunk = 1024;  // floats per CTA


__global__ void __launch_bounds__(kCommThreads) chpe_allreduce_residual_kernel(const CommPeers peers, int world, int rank,
                                                                          size_t slot_elems, int max_chunks,
                                                                          const float *__restrict__ part,
                                                                          float *__restrict__ hidden, int n,
                                                                          unsigned *__restrict__ ctr,
                                                                          volatile unsigned *host_failed,
                                                                          int *__restrict__ err) {
    __shared__ int s_ok;
    pdl_begin();  // the partial is the previous kernel's output
    const int c = blockIdx.x;
    // ctr[0] epoch, ctr[1] arrival ticket, ctr[2] failed mark
    if (*reinterpret_cast<volatile unsigned *>(&ctr[2])) {
        if (threadIdx.x == 0) atomicExch(err, kErrCommFailed);
        return;
    }
    const unsigned epoch = ctr[0] + 1u;  // ctr[0] advances only after every CTA of this launch read it
    if (threadIdx.x == 0) s_ok = 1;
    const int i0 = c * kCommChunk, i1 = min(n, i0 + kCommChunk);
    const size_t slot = ((size_t)(epoch & 1u) * world + rank) * slot_elems;
    // 2. push chunk c of this rank's partial to every peer, then raise the flags
    for (int r = 0; r < world; ++r) {
        if (r == rank) continue;
        float *dst = peers.recv[r] + slot;
        if (i1 - i0 == kCommChunk) {
            const float4 v = reinterpret_cast<const float4 *>(part + i0)[threadIdx.x];
            reinterpret_cast<float4 *>(dst + i0)[threadIdx.x] = v;
        } else {
            for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) dst[i] = part[i];
        }
    }
    __syncthreads();
    if (threadIdx.x < world && threadIdx.x != rank)
        st_release_sys(peers.flags[threadIdx.x] + (size_t)rank * max_chunks + c, epoch);
    // 3. wait for every peer's flag of this chunk (bounded)
    if (threadIdx.x < world && threadIdx.x != rank) {
        if (!wait_flag_bounded(peers.flags[rank] + (size_t)threadIdx.x * max_chunks + c, epoch)) {
            atomicExch(err, kErrCommWait);
            atomicExch(&ctr[2], 1u);  // failed: no later exchange on this object until a reset
            *host_failed = 1u;
            s_ok = 0;
        }
    }
    __syncthreads();
    if (s_ok) {
        // 4. hidden += sum of the partials in rank order
        const float *own = peers.recv[rank] + (size_t)(epoch & 1u) * world * slot_elems;
        for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
            float s = 0.0f;
            for (int r = 0; r < world; ++r) s += (r == rank) ? part[i] : own[(size_t)r * slot_elems + i];
            hidden[i] += s;
        }
    }
    // the last CTA to finish advances the epoch for the next all-reduce (not
    // after a failure: the object then stays failed until chpe_comm_reset)
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&ctr[1], 1u) == gridDim.x - 1) {
            ctr[1] = 0u;
            if (!atomicAdd(&ctr[2], 0u)) ctr[0] = epoch;
        }
    }
}

// The vocabulary-split LM head's argmax: every rank holds, for each of M
// rows, the (max value, index) of its shard; afterwards every rank holds the
// global pair -- the largest value, ties to the smaller global index, as
// src/engine.zig:1098-1110 computeArgmax breaks them within one shard.  One
// CTA, the same exchange protocol as the all-reduce on chunk 0 of the receive
// area (an exchange epoch of its own): thread m < M pushes row m's pair into
// slot [epoch & 1][rank] of every peer, thread r raises flag [rank][0] at peer
// r, waits (bounded) for peer r's flag, then thread m merges the pairs in rank
// order.  A slot is rewritten two epochs later only: the exchange between
// them needs every peer's flag, raised after that peer's previous kernel --
// the one that read the slot -- has finished (stream order).
__global__ void __launch_bounds__(32) chpe_argmax_merge_kernel(const CommPeers peers, int world, int rank,
                                                               size_t slot_elems, int max_chunks,
                                                               int *__restrict__ idx, float *__restrict__ maxv,
                                                               int M, int index_base, unsigned *__restrict__ ctr,
                                                               volatile unsigned *host_failed,
                                                               int *__restrict__ err) {
    __shared__ int s_ok;
    pdl_begin();  // the local argmax is the previous kernel's output
    if (*reinterpret_cast<volatile unsigned *>(&ctr[2])) {
        if (threadIdx.x == 0) atomicExch(err, kErrCommFailed);
        return;
    }
    const unsigned epoch = ctr[0] + 1u;
    const int m = threadIdx.x;
    if (m == 0) s_ok = 1;
    float v = 0.0f;
    int gi = 0;
    if (m < M) {
        v = maxv[m];
        gi = idx[m] + index_base;
    }
    const size_t slot = ((size_t)(epoch & 1u) * world + rank) * slot_elems;
    if (m < M)
        for (int r = 0; r < world; ++r) {
            if (r == rank) continue;
            reinterpret_cast<float2 *>(peers.recv[r] + slot)[m] = make_float2(v, __int_as_float(gi));
        }
    __syncthreads();
    if (m < world && m != rank) {
        st_release_sys(peers.flags[m] + (size_t)rank * max_chunks, epoch);
        if (!wait_flag_bounded(peers.flags[rank] + (size_t)m * max_chunks, epoch)) {
            atomicExch(err, kErrCommWait);
            atomicExch(&ctr[2], 1u);
            *host_failed = 1u;
            s_ok = 0;
        }
    }
    __syncthreads();
    if (s_ok && m < M) {
        const float2 *own = reinterpret_cast<const float2 *>(peers.recv[rank] + (size_t)(epoch & 1u) * world * slot_elems);
        float bv = 0.0f;
        int bi = 0;
        for (int r = 0; r < world; ++r) {
            float rv;
            int ri;
            if (r == rank) {
                rv = v;
                ri = gi;
            } else {
                const float2 q = own[(size_t)r * (slot_elems / 2) + m];
                rv = q.x;
                ri = __float_as_int(q.y);
            }
            if (r == 0 || rv > bv || (rv == bv && ri < bi)) {
                bv = rv;
                bi = ri;
            }
        }
        idx[m] = bi;
        maxv[m] = bv;
    }
    __syncthreads();
    if (m == 0 && !atomicAdd(&ctr[2], 0u)) ctr[0] = epoch;
}

}  // namespace
}  // namespace chpe

using namespace chpe;

struct chpe_comm {
    chpe_ctx *ctx = nullptr;
    int world = 0, rank = 0;
    size_t max_elems = 0;  // Mmax * H
    float *recv = nullptr;          // own receive area [2][world][max_elems]
    unsigned *flags = nullptr;      // own flags [world][max_chunks]
    unsigned *epoch = nullptr;      // own epoch counter, arrival ticket and failed mark
    unsigned *host_failed = nullptr;  // mapped pinned host word: set by a kernel whose wait expired
    unsigned *host_failed_dev = nullptr;
    int max_chunks = 0;
    CommPeers peers;
    bool opened[kCommMaxRanks] = {false};
    cudaIpcMemHandle_t handle_recv, handle_flags;
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
    c->max_chunks = (int)(c->max_elems / kCommChunk);
    memset(&c->peers, 0, sizeof c->peers);
    const size_t flag_bytes = (size_t)kCommMaxRanks * c->max_chunks * sizeof(unsigned);
    cudaError_t e = cudaMalloc(&c->recv, 2 * (size_t)world * c->max_elems * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&c->flags, flag_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&c->epoch, 256);
    if (e == cudaSuccess) e = cudaMemset(c->flags, 0, flag_bytes);
    if (e == cudaSuccess) e = cudaMemset(c->epoch, 0, 256);
    if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void **>(&c->host_failed), sizeof(unsigned),
                                            cudaHostAllocMapped);
    if (e == cudaSuccess) {
        *c->host_failed = 0u;
        e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&c->host_failed_dev), c->host_failed, 0);
    }
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&c->handle_recv, c->recv);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&c->handle_flags, c->flags);
    if (e != cudaSuccess) {
        cudaFree(c->recv);
        cudaFree(c->flags);
        cudaFree(c->epoch);
        if (c->host_failed) cudaFreeHost(c->host_failed);
        delete c;
        cudaGetLastError();
        return CHPE_ECUDA;
    }
    c->peers.recv[rank] = c->recv;
    c->peers.flags[rank] = c->flags;
    *out = c;
    return CHPE_OK;
}

extern "C" size_t chpe_comm_handle_bytes(void) { return 2 * sizeof(cudaIpcMemHandle_t); }

extern "C" int chpe_comm_handle(const chpe_comm *c, void *out) {
    if (!c || !out) return CHPE_EINVAL;
    memcpy(out, &c->handle_recv, sizeof(cudaIpcMemHandle_t));
    memcpy(static_cast<uint8_t *>(out) + sizeof(cudaIpcMemHandle_t), &c->handle_flags, sizeof(cudaIpcMemHandle_t));
    return CHPE_OK;
}

extern "C" int chpe_comm_open_peers(chpe_comm *c, const void *handles) {
    if (!c || !handles) return CHPE_EINVAL;
    const size_t hb = chpe_comm_handle_bytes();
    for (int r = 0; r < c->world; ++r) {
        if (r == c->rank || c->opened[r]) continue;
        cudaIpcMemHandle_t hr, hf;
        memcpy(&hr, static_cast<const uint8_t *>(handles) + r * hb, sizeof hr);
        memcpy(&hf, static_cast<const uint8_t *>(handles) + r * hb + sizeof hr, sizeof hf);
        void *pr = nullptr, *pf = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&pr, hr, cudaIpcMemLazyEnablePeerAccess);
        if (e == cudaSuccess) e = cudaIpcOpenMemHandle(&pf, hf, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            if (pr) cudaIpcCloseMemHandle(pr);
            cudaGetLastError();
            return CHPE_ECUDA;
        }
        c->peers.recv[r] = static_cast<float *>(pr);
        c->peers.flags[r] = static_cast<unsigned *>(pf);
        c->opened[r] = true;
    }
    return CHPE_OK;
}

extern "C" int chpe_allreduce_residual_dev(chpe_comm *c, const float *part, float *hidden, size_t n, void *stream) {
    if (!c || !part || !hidden) return CHPE_EINVAL;
    if (n > c->max_elems) return CHPE_EINVAL;
    if (reinterpret_cast<uintptr_t>(part) % 16) return CHPE_EALIGN;  // read as float4
    for (int r = 0; r < c->world; ++r)
        if (!c->peers.recv[r] || !c->peers.flags[r]) return CHPE_ENOENT;  // peers not opened yet
    // a failed object (a bounded wait expired) takes no exchange until chpe_comm_reset
    if (*reinterpret_cast<volatile unsigned *>(c->host_failed)) return CHPE_ETIMEOUT;
    if (n == 0) return CHPE_OK;
    const unsigned chunks = (unsigned)((n + kCommChunk - 1) / kCommChunk);
    cudaError_t e = launch_pdl(chpe_allreduce_residual_kernel, dim3(chunks), dim3(kCommThreads), 0,
                               static_cast<cudaStream_t>(stream), c->peers, c->world, c->rank, c->max_elems,
                               c->max_chunks, part, hidden, (int)n, c->epoch, c->host_failed_dev,
                               chpe_ctx_error_word(c->ctx));
    return e == cudaSuccess ? CHPE_OK : CHPE_ECUDA;
}

extern "C" int chpe_argmax_merge_dev(chpe_comm *c, int *idx, float *maxv, int M, int index_base, void *stream) {
    if (!c || !idx || !maxv) return CHPE_EINVAL;
    if (M < 1 || M > 32 || (size_t)2 * M > c->max_elems) return CHPE_EINVAL;
    for (int r = 0; r < c->world; ++r)
        if (!c->peers.recv[r] || !c->peers.flags[r]) return CHPE_ENOENT;
    if (*reinterpret_cast<volatile unsigned *>(c->host_failed)) return CHPE_ETIMEOUT;
    cudaError_t e = launch_pdl(chpe_argmax_merge_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream),
                               c->peers, c->world, c->rank, c->max_elems, c->max_chunks, idx, maxv, M, index_base,
                               c->epoch, c->host_failed_dev, chpe_ctx_error_word(c->ctx));
    return e == cudaSuccess ? CHPE_OK : CHPE_ECUDA;
}

// The exchange state a fused fill needs (launch_xfill_f16): refuses like
// chpe_allreduce_residual_dev, and with CHPE_ENOTSUP when n partials do not
// fit the receive area.
int comm_fill_exchange(chpe_comm *c, const float *part, float *hidden, size_t n, FillExchange *out) {
    if (!c || !part || !hidden || !out) return CHPE_EINVAL;
    if (n > c->max_elems) return CHPE_ENOTSUP;
    for (int r = 0; r < c->world; ++r)
        if (!c->peers.recv[r] || !c->peers.flags[r]) return CHPE_ENOENT;
    if (*reinterpret_cast<volatile unsigned *>(c->host_failed)) return CHPE_ETIMEOUT;
    FillExchange ex;
    ex.peers = c->peers;
    ex.world = c->world;
    ex.rank = c->rank;
    ex.slot_elems = c->max_elems;
    ex.max_chunks = c->max_chunks;
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
    const size_t flag_bytes = (size_t)kCommMaxRanks * c->max_chunks * sizeof(unsigned);
    if (e == cudaSuccess) e = cudaMemset(c->flags, 0, flag_bytes);
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
    for (int r = 0; r < c->world; ++r) {
        if (!c->opened[r]) continue;
        cudaIpcCloseMemHandle(c->peers.recv[r]);
        cudaIpcCloseMemHandle(c->peers.flags[r]);
    }
    cudaFree(c->recv);
    cudaFree(c->flags);
    cudaFree(c->epoch);
    cudaFreeHost(c->host_failed);
    delete c;
    return CHPE_OK;
}
