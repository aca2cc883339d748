// ep.cuh: the device side of expert parallelism. Experts are placed E / N per GPU; every rank routes its own tokens
// (the router is replicated), sends each (token, slot) row to the rank that holds its expert, and sums the returned
// expert outputs in increasing expert id.
//
//  pack     a stable counting sort of the rank's (token, slot) rows by destination rank, and the rows and expert ids
//           in that order (the send buffer of an all-to-all).
//  experts  the expert FFN of rows that arrive in any order, each with its expert id: a stable counting sort by
//           expert, the grouped gate / up products, SwiGLU, the grouped down product (the kernel-level kernels of
//           kernel_api.cuh, the same exact definitions as the layer kernels), the outputs back in arrival order.
//  combine  prefill.cuh's trx_k_pf_combine over the returned rows (the send order's place of each row).
// Every row's arithmetic is the one-GPU road's, so the layer's output is bit for bit the one-GPU output.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "kernel_api.cuh"

// Stable counting sort of n keys into nk <= 64 buckets by one block of 1024 threads (32 warps, each a contiguous
// chunk of j). key(j) = src64 ? src64[j] / div : src32[j]. Writes offsets[0..nk], place[j] (the row's position in
// bucket order), xmap[place[j]] = j, and counts[b] when counts is not NULL.
__global__ void __launch_bounds__(1024) trx_k_stable_sort(const int64_t *__restrict__ src64, const int32_t *__restrict__ src32,
                                                          int64_t div, int n, int nk, int32_t *__restrict__ offsets,
                                                          int32_t *__restrict__ place, int32_t *__restrict__ xmap,
                                                          int32_t *__restrict__ counts) {
    __shared__ int wc[32][64];
    __shared__ int tot[65];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int chunk = (n + 31) / 32, j0 = warp * chunk, j1 = min(n, j0 + chunk);
    for (int e = lane; e < 64; e += 32) wc[warp][e] = 0;
    __syncwarp();
    auto key = [&](int j) { // a key out of range is dropped (no row of ours carries one)
        const int k = src64 ? (int)(src64[j] / div) : src32[j];
        return k >= 0 && k < nk ? k : -1;
    };
    for (int b = j0; b < j1; b += 32) {
        const int j = b + lane;
        const int k = j < j1 ? key(j) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, k);
        if (k >= 0 && lane == __ffs(peers) - 1) wc[warp][k] += __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    if (tid < 64) { // bucket tid: its total, and each warp's exclusive start within the bucket
        int s = 0;
        for (int w = 0; w < 32; w++) {
            const int c = wc[w][tid];
            wc[w][tid] = s;
            s += c;
        }
        tot[tid] = tid < nk ? s : 0;
    }
    __syncthreads();
    if (tid == 0) {
        int s = 0;
        for (int e = 0; e < nk; e++) {
            const int c = tot[e];
            tot[e] = s;
            s += c;
        }
        tot[nk] = s;
    }
    __syncthreads();
    if (tid <= nk) offsets[tid] = tot[tid];
    if (counts && tid < nk) counts[tid] = tot[tid + 1] - tot[tid];
    if (tid < 64)
        for (int w = 0; w < 32; w++) wc[w][tid] += tot[tid];
    __syncthreads();
    for (int b = j0; b < j1; b += 32) {
        const int j = b + lane;
        const int k = j < j1 ? key(j) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, k);
        if (k >= 0) {
            const int pos = wc[warp][k] + __popc(peers & ((1u << lane) - 1u));
            place[j] = pos;
            xmap[pos] = j;
        }
        __syncwarp();
        if (k >= 0 && lane == __ffs(peers) - 1) wc[warp][k] += __popc(peers);
        __syncwarp();
    }
}

// dst row pos = src row xmap[pos] / div (cols floats, cols % 4 == 0); ids_out[pos] = ids_in[xmap[pos]] when given.
// Rows past *n_sorted (the sort's total: rows with a dropped key) are not touched. cap > 0 (the pack's padded form):
// the rows of bucket b = ids_in[j] / kdiv go to b cap + their rank in the bucket instead, and place[j] says so.
__global__ void __launch_bounds__(256) trx_k_gather_rows(const float *__restrict__ src, const int32_t *__restrict__ xmap,
                                                         const int32_t *__restrict__ n_sorted, int div, int cols,
                                                         float *__restrict__ dst, const int64_t *__restrict__ ids_in,
                                                         int32_t *__restrict__ ids_out, const int32_t *__restrict__ offsets,
                                                         int cap, int64_t kdiv, int32_t *__restrict__ place) {
    const int pos = blockIdx.x;
    if (pos >= *n_sorted) return;
    const int j = xmap[pos];
    int dpos = pos;
    if (cap > 0) {
        const int b = (int)(ids_in[j] / kdiv);
        dpos = b * cap + pos - offsets[b];
        if (threadIdx.x == 0) place[j] = dpos;
    }
    const float4 *s = reinterpret_cast<const float4 *>(src + (int64_t)(j / div) * cols);
    float4 *d = reinterpret_cast<float4 *>(dst + (int64_t)dpos * cols);
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) d[i] = s[i];
    if (ids_out && threadIdx.x == 0) ids_out[dpos] = (int32_t)ids_in[j];
}

// out row xmap[pos] = src row pos, for pos < *n_sorted
__global__ void __launch_bounds__(256) trx_k_scatter_rows(const float *__restrict__ src, const int32_t *__restrict__ xmap,
                                                          const int32_t *__restrict__ n_sorted, int cols,
                                                          float *__restrict__ out) {
    const int pos = blockIdx.x;
    if (pos >= *n_sorted) return;
    const float4 *s = reinterpret_cast<const float4 *>(src + (int64_t)pos * cols);
    float4 *d = reinterpret_cast<float4 *>(out + (int64_t)xmap[pos] * cols);
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) d[i] = s[i];
}

// ---------------------------------------------------------------------------------------------
// Expert parallelism over peer memory (NVLink stores, no NCCL on the data path). Every rank's exchange region holds,
// for n sources of cap rows each: the rows and expert ids it receives, the output rows returned to it, and one
// arrival flag per source for each direction. A step's epoch (the rank's step count, the same on every rank) tells
// the flags of this step from older ones. Every wait is bounded; a rank that gives up sets the error flag.

#define TRX_EP_MAX_RANKS 64
#define TRX_EP_WAIT_NS 10000000000ull // the waits on other ranks: bounded, and above the host skew of test ranks

struct TrxEpHdr {
    uint32_t epoch;                         // this rank's steps so far (the dispatch advances it)
    uint32_t pad[31];
    uint32_t recv_flag[TRX_EP_MAX_RANKS];   // source s's rows of step `epoch` have arrived
    uint32_t back_flag[TRX_EP_MAX_RANKS];   // owner d's output rows of step `epoch` have arrived
};

struct TrxEpPeers {
    int n, rank, cap, H;
    size_t off_ids, off_rows, off_back;     // within a region: ids [n][cap], rows [n][cap][H], returned rows [n][cap][H]
    uint8_t *base[TRX_EP_MAX_RANKS];        // every rank's region as this GPU addresses it (its own included)
};

__host__ __device__ inline void trx_ep_layout(int n, int cap, int H, size_t &ids, size_t &rows, size_t &back,
                                              size_t &total) {
    ids = (sizeof(TrxEpHdr) + 255) / 256 * 256;
    rows = (ids + (size_t)n * cap * 4 + 255) / 256 * 256;
    back = rows + (size_t)n * cap * H * 4;
    total = back + (size_t)n * cap * H * 4;
}

__device__ __forceinline__ uint32_t trx_ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// a flag in another GPU's memory: a system-scope atomic exchange with release semantics, performed at the memory's
// own GPU (a plain store to a peer can stay in flight; the atomic is carried out where the flag lives)
// (returns the flag's previous value)
__device__ __forceinline__ uint32_t trx_st_release_sys(uint32_t *p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.release.sys.global.exch.b32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Waits until flags[0..n) all hold `epoch` (one thread); false when it gave up (limit_ns after the first flag it
// found unset), with *why = the source it waited for, the value it last saw and the epoch it wanted, packed for the
// error flag
__device__ inline bool trx_ep_wait_flags(const uint32_t *flags, int n, uint32_t epoch, uint64_t limit_ns, int *why) {
    uint64_t t0 = 0;
    bool timing = false; // the clock starts at the first miss, whichever flag it is on
    for (int s = 0; s < n;) {
        const uint32_t v = trx_ld_acquire_sys(flags + s);
        if (v == epoch) {
            s++;
            continue;
        }
        uint64_t now;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
        if (!timing) {
            t0 = now;
            timing = true;
        } else if (now - t0 > limit_ns) {
            *why = (s & 15) << 4 | (int)(v & 0xfffu) << 8 | (int)(epoch & 0x7ffu) << 20;
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// The dispatch (one block of 256 threads, R = T k <= cap rows): this rank's (token, slot) rows and their expert ids
// straight into their owner's region, at [this rank][the row's rank among this rank's rows to that owner] (stable:
// increasing j), the unused slots' ids -1; then, after a system-scope fence, every owner's arrival flag. place[j]:
// where row j's output comes back (owner d, slot q: d cap + q). Advances the step's epoch.
__global__ void __launch_bounds__(256) trx_k_ep_dispatch(const int64_t *__restrict__ sel_id, int T, int k, int per_rank,
                                                         const float *__restrict__ normed, const TrxEpPeers *__restrict__ P,
                                                         int32_t *__restrict__ place) {
    __shared__ int s_dst[256], s_pos[256], s_cnt[TRX_EP_MAX_RANKS];
    __shared__ uint32_t s_epoch;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, R = T * k, n = P->n, rank = P->rank, cap = P->cap,
              H = P->H;
    TrxEpHdr *own = reinterpret_cast<TrxEpHdr *>(P->base[rank]);
    if (tid == 0) {
        s_epoch = own->epoch + 1u;
        own->epoch = s_epoch;
    }
    if (tid < TRX_EP_MAX_RANKS) s_cnt[tid] = 0;
    __syncthreads();
    if (tid == 0) // R <= 256 rows: a serial stable count is cheap
        for (int j = 0; j < R; j++) {
            const int d = (int)(sel_id[j] / per_rank);
            s_dst[j] = d;
            s_pos[j] = s_cnt[d]++;
            place[j] = d * cap + s_pos[j];
        }
    __syncthreads();
    for (int j = warp; j < R; j += blockDim.x / 32) { // a warp a row
        const int d = s_dst[j], q = rank * cap + s_pos[j];
        const float4 *src = reinterpret_cast<const float4 *>(normed + (int64_t)(j / k) * H);
        float4 *dst = reinterpret_cast<float4 *>(P->base[d] + P->off_rows + (size_t)q * H * 4);
        for (int i = lane; i < H / 4; i += 32) dst[i] = src[i];
        if (lane == 0) reinterpret_cast<int32_t *>(P->base[d] + P->off_ids)[q] = (int32_t)sel_id[j];
    }
    for (int i = tid; i < n * cap; i += blockDim.x) { // the unused slots of every owner: no expert
        const int d = i / cap, q = i % cap;
        if (q >= s_cnt[d]) reinterpret_cast<int32_t *>(P->base[d] + P->off_ids)[rank * cap + q] = -1;
    }
    __threadfence_system(); // every thread's rows and ids, before the flags
    __syncthreads();
    if (tid < n) trx_st_release_sys(&reinterpret_cast<TrxEpHdr *>(P->base[tid])->recv_flag[rank], s_epoch);
}

// The combine of the returned rows: waits (one thread a block) for every owner's return flag of this step, then x[t]
// += sum over slots in expert-id order of w * back[place] (and ffn_out), as trx_k_pf_combine
__global__ void __launch_bounds__(256) trx_k_ep_peer_combine(const float *__restrict__ sel_w, const int32_t *__restrict__ place,
                                                             const TrxEpPeers *__restrict__ P, int T, int k,
                                                             float *__restrict__ x, float *__restrict__ ffn_out,
                                                             int32_t *__restrict__ err) {
    __shared__ int s_ok;
    const TrxEpHdr *own = reinterpret_cast<const TrxEpHdr *>(P->base[P->rank]);
    if (threadIdx.x == 0) {
        int why = 0;
        s_ok = trx_ep_wait_flags(own->back_flag, P->n, own->epoch, TRX_EP_WAIT_NS, &why);
        if (!s_ok) atomicCAS(err, 0, 6 | why); // the first error stays
    }
    __syncthreads();
    if (!s_ok) return;
    const int H = P->H;
    const float *back = reinterpret_cast<const float *>(P->base[P->rank] + P->off_back);
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * H) return;
    const int t = (int)(i / H), d = (int)(i % H);
    float out = 0.0f;
    for (int s = 0; s < k; s++)
        out = __fadd_rn(out, __fmul_rn(sel_w[t * k + s], back[(int64_t)place[t * k + s] * H + d]));
    if (ffn_out) ffn_out[i] = out;
    x[i] = __fadd_rn(x[i], out);
}
