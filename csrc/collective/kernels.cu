// Collectives on ugdr's memory model: every rank's buffers are CUDA-IPC mapped into every other
// rank's process (the same export / open path as MR registration), and sm_100a kernels move the
// data with direct NVLink loads and stores, fusing the arithmetic into the transfer.
//
//  * Allreduce (bf16, fp32 accumulation), one kernel: rank r pulls shard r from every rank, sums,
//    and pushes the sum into every rank's buffer, vector by vector.  2 (N - 1) / N of the buffer
//    crosses NVLink per GPU, the ring optimum, with both link directions busy throughout.
//  * MoE routing (moe_route): deterministic counting sort of (token, k) rows by expert - counts per
//    expert and each row's position within its expert group.  Scratch: per-block histograms.
//  * MoE dispatch: each (token, k) row is stored straight into the expert owner's receive
//    buffer at [expert group base + position], i.e. the permute is the NVLink store itself.
//  * MoE combine: each token pulls its top-k expert rows back over NVLink and applies the routing
//    weights in fp32: the unpermute and the weighted reduction are the NVLink load itself.
//
// Cross-GPU ordering: a kernel that must not return before every peer finished the same phase
// ends with an arrival counter; the last CTA to arrive publishes `epoch` into each peer's signal
// word (st.release.sys) and waits, with a %globaltimer bound, until every peer's word for this
// rank reaches `epoch`.  Only that one CTA waits, so no co-residency is assumed; kernels on
// different GPUs run concurrently by construction.  A wait that runs out sets *status and returns.
#include "collective/kernels.hpp"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ugdr::coll {
namespace {

__device__ __forceinline__ uint64_t gtime() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint64_t ld_acq_sys(const void *p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_rel_sys(void *p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint4 ld128(const void *p) {
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ void st128(void *p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Last-arriving CTA signals every peer and waits for theirs.  Called by every thread of every CTA.
__device__ void end_barrier(const PeerSet &ps, uint64_t epoch, uint32_t slot, uint64_t max_ns) {
    __syncthreads();
    if (threadIdx.x != 0) return;
    __threadfence_system();
    unsigned int *arrive = &ps.arrive[slot];
    const unsigned int old = atomicAdd(arrive, 1u);
    if (old + 1 != gridDim.x) return;
    atomicExch(arrive, 0u);  // re-arm for the next launch (stream order separates launches)
    // Signal word layout in every rank's signal buffer: sig[slot * kMaxRanks + sender].
    for (int q = 0; q < ps.n; ++q) {
        uint64_t *w = ps.signal[q] + slot * kMaxRanks + ps.rank;
        st_rel_sys(w, epoch);
    }
    const uint64_t *mine = ps.signal[ps.rank] + slot * kMaxRanks;
    const uint64_t t0 = gtime();
    for (int q = 0; q < ps.n; ++q) {
        uint32_t spins = 0;
        while (ld_acq_sys(mine + q) < epoch) {
            if ((++spins & 255) == 0 && gtime() - t0 > max_ns) {
                atomicExch(ps.status, 1u);
                return;
            }
            __nanosleep(64);
        }
    }
}

__device__ __forceinline__ void acc8(float (&a)[8], uint4 v) {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        a[2 * i] += f.x;
        a[2 * i + 1] += f.y;
    }
}
__device__ __forceinline__ uint4 pack8(const float (&a)[8]) {
    uint4 v;
    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
    return v;
}

// ---- allreduce ---------------------------------------------------------------------------------

// Entry handshake: every CTA's thread 0 publishes `epoch` into each peer's entry word for this
// rank and waits (bounded) until every peer's word in its own signal buffer reached `epoch`, i.e.
// every rank has launched this call, so its input is in place and its previous call is over.
// The waits read local memory only; peers' kernels run on other GPUs, so no co-residency is
// assumed.
__device__ void entry_barrier(const PeerSet &ps, uint64_t epoch, uint32_t slot, uint64_t max_ns) {
    if (threadIdx.x == 0) {
        for (int q = 0; q < ps.n; ++q) st_rel_sys(ps.signal[q] + slot * kMaxRanks + ps.rank, epoch);
        const uint64_t *mine = ps.signal[ps.rank] + slot * kMaxRanks;
        const uint64_t t0 = gtime();
        for (int q = 0; q < ps.n; ++q) {
            uint32_t spins = 0;
            while (ld_acq_sys(mine + q) < epoch) {
                if ((++spins & 255) == 0 && gtime() - t0 > max_ns) {
                    atomicExch(ps.status, 1u);
                    break;
                }
                __nanosleep(32);
            }
        }
    }
    __syncthreads();
}

// One-kernel allreduce.  Rank r owns shard r of the buffer; for each 16-byte vector of it a
// thread loads the vector from every rank (NVLink loads), sums in fp32, rounds to bf16 once, and
// stores the result into every rank's buffer (NVLink stores).  Shard r of a peer's buffer is
// read and written only by rank r, and a thread reads an element before it overwrites it, so no
// barrier is needed between the reduce and the broadcast: they overlap vector by vector, and
// both link directions carry traffic for the whole kernel.  Per GPU, (N - 1) / N of the buffer
// arrives by loads and (N - 1) / N by peers' stores: 2 (N - 1) / N in total, the ring optimum.
template <int NR>
__global__ void __launch_bounds__(512) allreduce_kernel(PeerSet ps, uint64_t base_off, uint64_t nvec,
                                                        uint64_t epoch, uint64_t max_ns) {
    entry_barrier(ps, epoch, kSlotArEntry, max_ns);
    const uint64_t per = (nvec + ps.n - 1) / ps.n;
    const uint64_t begin = min(nvec, per * ps.rank), end = min(nvec, begin + per);
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    uint8_t *bufs[NR];
#pragma unroll
    for (int q = 0; q < NR; ++q)
        bufs[q] = q < ps.n ? reinterpret_cast<uint8_t *>(ps.buf[q]) + base_off : nullptr;
    for (uint64_t i = begin + blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < end; i += 2 * stride) {
        const bool two = i + stride < end;
        uint4 va[NR], vb[NR];
#pragma unroll
        for (int q = 0; q < NR; ++q) {
            if (q < ps.n) {
                va[q] = ld128(bufs[q] + i * 16);
                if (two) vb[q] = ld128(bufs[q] + (i + stride) * 16);
            }
        }
        // Each vector is summed once, by its owner, in rank order, and the same bits go to every
        // rank.
        float a[8] = {0, 0, 0, 0, 0, 0, 0, 0}, b[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int q = 0; q < NR; ++q) {
            if (q < ps.n) {
                acc8(a, va[q]);
                if (two) acc8(b, vb[q]);
            }
        }
        const uint4 ra = pack8(a), rb = pack8(b);
#pragma unroll
        for (int q = 0; q < NR; ++q) {
            if (q < ps.n) {
                st128(bufs[q] + i * 16, ra);
                if (two) st128(bufs[q] + (i + stride) * 16, rb);
            }
        }
    }
    end_barrier(ps, epoch, kSlotArEnd, max_ns);
}

// NVLS allreduce: rank r owns shard r; for each 16-byte vector of it, one multimem.ld_reduce
// through the multicast view has the NVSwitch read the vector from every GPU and return the
// fp32-accumulated bf16 sum, and one multimem.st writes the sum to every GPU.  Per GPU about
// (1 + 1/N) of the buffer crosses each link direction instead of 2 (N - 1) / N.  Peer data is
// read only through the multicast alias, so a proxy fence after the entry handshake orders the
// peers' unicast writes of their inputs before the reads, and one before the exit barrier orders
// the multicast stores before the peers' unicast reads of the result.
__device__ __forceinline__ uint4 mm_ld_add_bf16x8(const uint8_t *p) {
    uint4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ void mm_st_bf16x8(uint8_t *p, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

template <int U>
__global__ void __launch_bounds__(512) allreduce_nvls_kernel(PeerSet ps, uint8_t *mc, uint64_t nvec, uint64_t epoch,
                                                             uint64_t max_ns) {
    entry_barrier(ps, epoch, kSlotArEntry, max_ns);
    asm volatile("fence.proxy.alias;" ::: "memory");
    const uint64_t per = (nvec + ps.n - 1) / ps.n;
    const uint64_t begin = min(nvec, per * ps.rank), end = min(nvec, begin + per);
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = begin + blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < end; i += U * stride) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i + u * stride < end) v[u] = mm_ld_add_bf16x8(mc + (i + u * stride) * 16);
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (i + u * stride < end) mm_st_bf16x8(mc + (i + u * stride) * 16, v[u]);
    }
    asm volatile("fence.proxy.alias;" ::: "memory");
    end_barrier(ps, epoch, kSlotArEnd, max_ns);
}

// ---- MoE routing (counting sort) ---------------------------------------------------------------

// K1: per-block expert histogram of rows [b * R, (b + 1) * R).
__global__ void route_hist_kernel(const int32_t *idx, uint64_t rows, int nexp, uint32_t *hist) {
    extern __shared__ uint32_t sh[];
    for (int e = threadIdx.x; e < nexp; e += blockDim.x) sh[e] = 0;
    __syncthreads();
    const uint64_t b0 = uint64_t(blockIdx.x) * kRouteRowsPerBlock;
    const uint64_t b1 = min(rows, b0 + kRouteRowsPerBlock);
    for (uint64_t r = b0 + threadIdx.x; r < b1; r += blockDim.x) {
        const int e = idx[r];
        if (e >= 0 && e < nexp) atomicAdd(&sh[e], 1u);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nexp; e += blockDim.x) hist[uint64_t(blockIdx.x) * nexp + e] = sh[e];
}

// K2: per expert, exclusive scan over blocks (in place: hist becomes block offsets) + totals.
__global__ void route_scan_kernel(uint32_t *hist, int nblocks, int nexp, int32_t *counts) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= nexp) return;
    uint32_t run = 0;
    for (int b = 0; b < nblocks; ++b) {
        const uint32_t c = hist[uint64_t(b) * nexp + e];
        hist[uint64_t(b) * nexp + e] = run;
        run += c;
    }
    counts[e] = int32_t(run);
}

// K3: positions in row order.  The block first stages its rows' expert ids in shared memory
// (all threads, coalesced), then one warp walks them 32 at a time and ranks equal experts with
// __match_any_sync, so the result is deterministic and the walk costs no global round trips.
__global__ void route_place_kernel(const int32_t *idx, uint64_t rows, int nexp, const uint32_t *off,
                                   int32_t *pos) {
    extern __shared__ uint32_t cur[];
    __shared__ int32_t ids[kRouteRowsPerBlock];
    const uint64_t b0 = uint64_t(blockIdx.x) * kRouteRowsPerBlock;
    const uint64_t b1 = min(rows, b0 + kRouteRowsPerBlock);
    const int n = int(b1 - b0);
    for (int e = threadIdx.x; e < nexp; e += blockDim.x) cur[e] = off[uint64_t(blockIdx.x) * nexp + e];
    for (int i = threadIdx.x; i < n; i += blockDim.x) ids[i] = idx[b0 + i];
    __syncthreads();
    const int lane = threadIdx.x;
    for (int i0 = 0; threadIdx.x < 32 && i0 < n; i0 += 32) {
        const int i = i0 + lane;
        const bool live = i < n;
        int e = live ? ids[i] : -1;
        const bool ok = live && e >= 0 && e < nexp;
        if (!ok) e = -1 - lane;  // unique key: never matches a real expert or another lane
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const unsigned lower = same & ((1u << lane) - 1);
        const uint32_t base = ok ? cur[e] : 0;
        __syncwarp();
        if (ok && lower == 0) cur[e] = base + __popc(same);
        __syncwarp();
        if (live) ids[i] = ok ? int32_t(base + __popc(lower)) : -1;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) pos[b0 + i] = ids[i];
}

// ---- MoE dispatch / combine --------------------------------------------------------------------

// Row resolution shared by dispatch and combine: lane j of the warp resolves row r0 + j (its
// expert, owner and row in the owner's receive area) in one round of parallel loads; the copy
// loops then take the pointers by shuffle, so no dependent index loads sit between row copies.
struct RowRef {
    uint8_t *ptr;  // the row in its owner's receive area (null: skipped)
    float w;
};

__device__ __forceinline__ RowRef resolve_row(const PeerSet &ps, const int32_t *idx, const int32_t *pos,
                                              const int64_t *gbase, const float *w, uint64_t r, bool live,
                                              int exp_per_rank, uint64_t recv_off, uint64_t recv_rows,
                                              uint64_t row_bytes) {
    RowRef ref{nullptr, 0.f};
    if (!live) return ref;
    const int e = idx[r];
    const int p = pos[r];
    if (w != nullptr) ref.w = w[r];
    if (e < 0 || p < 0) return ref;
    const int owner = e / exp_per_rank;
    const uint64_t row = uint64_t(gbase[e]) + uint64_t(p);
    if (owner >= ps.n || row >= recv_rows) {
        atomicExch(ps.status, 2u);  // receive buffer too small: recorded, row skipped
        return ref;
    }
    ref.ptr = reinterpret_cast<uint8_t *>(ps.buf[owner]) + recv_off + row * row_bytes;
    return ref;
}

// 32-byte vector loads / stores (sm_100 256-bit global accesses).
struct alignas(32) V256 {
    uint32_t w[8];
};
__device__ __forceinline__ V256 ld256(const void *p) {
    V256 v;
    asm volatile("ld.global.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                   "=r"(v.w[6]), "=r"(v.w[7])
                 : "l"(p));
    return v;
}
__device__ __forceinline__ void st256(void *p, const V256 &v) {
    asm volatile("st.global.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]),
                 "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]), "r"(v.w[7])
                 : "memory");
}

// One row copied by a warp: 32-byte vectors (4 in flight per lane) when both ends and the length
// are 32-byte aligned, else 16-byte vectors (8 in flight).
__device__ __forceinline__ void warp_copy_row(uint8_t *dst, const uint8_t *src, uint64_t bytes, int lane) {
    if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | bytes) & 31) == 0) {
        const uint64_t nv = bytes / 32;
        uint64_t i = lane;
        for (; i + 3 * 32 < nv; i += 4 * 32) {
            V256 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = ld256(src + (i + u * 32) * 32);
#pragma unroll
            for (int u = 0; u < 4; ++u) st256(dst + (i + u * 32) * 32, v[u]);
        }
        for (; i < nv; i += 32) st256(dst + i * 32, ld256(src + i * 32));
        return;
    }
    const uint64_t nv = bytes / 16;
    uint64_t i = lane;
    for (; i + 7 * 32 < nv; i += 8 * 32) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = ld128(src + (i + u * 32) * 16);
#pragma unroll
        for (int u = 0; u < 8; ++u) st128(dst + (i + u * 32) * 16, v[u]);
    }
    for (; i < nv; i += 32) st128(dst + i * 16, ld128(src + i * 16));
}

// Dispatch: row (t, k) -> recv buffer of the expert's owner at row gbase[e] + pos[(t, k)]
// (`gbase[e]` = first row of expert e's group in its owner's buffer for rows of THIS rank).
// Rows are interleaved over all warps of the grid (warp w takes rows w, w + W, ...), so work
// stays balanced whatever the row count; each warp resolves its next 32 rows lane-parallel in
// one round of loads, then copies them one by one.
__global__ void __launch_bounds__(512) dispatch_kernel(PeerSet ps, const uint8_t *x, uint64_t row_bytes,
                                                       const int32_t *idx, const int32_t *pos,
                                                       const int64_t *gbase, uint64_t rows, int topk,
                                                       int exp_per_rank, uint64_t recv_off, uint64_t recv_rows,
                                                       uint64_t epoch, uint64_t max_ns) {
    const int lane = threadIdx.x & 31;
    const uint64_t warp = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
    for (uint64_t base = warp; base < rows; base += 32 * nwarps) {
        const uint64_t mine_row = base + uint64_t(lane) * nwarps;
        const RowRef mine = resolve_row(ps, idx, pos, gbase, nullptr, mine_row, mine_row < rows, exp_per_rank,
                                        recv_off, recv_rows, row_bytes);
        for (int j = 0; j < 32; ++j) {
            const uint64_t r = base + uint64_t(j) * nwarps;
            if (r >= rows) break;
            uint8_t *dst = reinterpret_cast<uint8_t *>(
                __shfl_sync(0xffffffffu, reinterpret_cast<uint64_t>(mine.ptr), j));
            if (dst == nullptr) continue;
            warp_copy_row(dst, x + (r / topk) * row_bytes, row_bytes, lane);
        }
    }
    end_barrier(ps, epoch, kSlotDispatch, max_ns);
}

// Combine: out[t] = sum_k w[t, k] * expert_out_row(t, k), rows pulled from their owners.  Lane
// k (< topk) resolves row (t, k); every lane then streams its 16-byte columns with all top-k
// loads of a column (two columns per step) in flight before the fp32 weighted sum.
template <int TOPK>
__global__ void __launch_bounds__(512) combine_kernel(PeerSet ps, uint8_t *out, uint64_t row_bytes,
                                                      const int32_t *idx, const int32_t *pos,
                                                      const int64_t *gbase, const float *w, uint64_t ntok,
                                                      int topk, int exp_per_rank, uint64_t recv_off,
                                                      uint64_t recv_rows, uint64_t epoch, uint64_t max_ns) {
    const int lane = threadIdx.x & 31;
    const uint64_t warp = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
    const uint64_t nv = row_bytes / 16;
    for (uint64_t t = warp; t < ntok; t += nwarps) {
        const RowRef mine = resolve_row(ps, idx, pos, gbase, w, t * topk + lane, lane < topk, exp_per_rank,
                                        recv_off, recv_rows, row_bytes);
        const uint8_t *sp[TOPK];
        float wk[TOPK];
#pragma unroll
        for (int k = 0; k < TOPK; ++k) {
            sp[k] = reinterpret_cast<const uint8_t *>(
                __shfl_sync(0xffffffffu, reinterpret_cast<uint64_t>(mine.ptr), k));
            wk[k] = __shfl_sync(0xffffffffu, mine.w, k);
        }
        uint8_t *orow = out + t * row_bytes;
        constexpr uint64_t kStep = TOPK <= 8 ? 64 : 32;  // two columns per step while registers allow
        for (uint64_t i = lane; i < nv; i += kStep) {
            const bool two = kStep == 64 && i + 32 < nv;
            uint4 va[TOPK], vb[TOPK];
#pragma unroll
            for (int k = 0; k < TOPK; ++k) {
                if (sp[k] != nullptr) {
                    va[k] = ld128(sp[k] + i * 16);
                    if (two) vb[k] = ld128(sp[k] + (i + 32) * 16);
                }
            }
            float a[8] = {0, 0, 0, 0, 0, 0, 0, 0}, b[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int k = 0; k < TOPK; ++k) {
                if (sp[k] == nullptr) continue;
                float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                acc8(f, va[k]);
#pragma unroll
                for (int j = 0; j < 8; ++j) a[j] += wk[k] * f[j];
                if (two) {
                    float g[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                    acc8(g, vb[k]);
#pragma unroll
                    for (int j = 0; j < 8; ++j) b[j] += wk[k] * g[j];
                }
            }
            st128(orow + i * 16, pack8(a));
            if (two) st128(orow + (i + 32) * 16, pack8(b));
        }
    }
    end_barrier(ps, epoch, kSlotCombine, max_ns);
}

// Weighted sum of rows that are already local, in (token, k) order (the combine of the MoE
// all-to-all on the verbs, whose READs brought the rows back): out[t] = sum_k w[t, k] * rows[t, k],
// fp32 accumulation.  One warp per token; every lane keeps all top-k loads of its columns in
// flight before the sum.
template <int TOPK>
__global__ void __launch_bounds__(512) weighted_rows_kernel(uint8_t *out, const uint8_t *rows, const float *w,
                                                            uint64_t ntok, int topk, uint64_t row_bytes,
                                                            const int32_t *ids, const int32_t *pos,
                                                            const int64_t *start) {
    const int lane = threadIdx.x & 31;
    const uint64_t warp = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
    const uint64_t nv = row_bytes / 16;
    for (uint64_t t = warp; t < ntok; t += nwarps) {
        float wk[TOPK];
#pragma unroll
        for (int k = 0; k < TOPK; ++k) wk[k] = k < topk ? __ldg(w + t * topk + k) : 0.f;
        // Row (t, k): at t * topk + k, or (grouped) at start[expert] + position.
        const uint8_t *rk[TOPK];
#pragma unroll
        for (int k = 0; k < TOPK; ++k) {
            uint64_t row = t * uint64_t(topk) + uint64_t(k);
            if (ids != nullptr && k < topk) row = uint64_t(__ldg(start + __ldg(ids + row))) + uint64_t(__ldg(pos + row));
            rk[k] = rows + row * row_bytes;
        }
        uint8_t *orow = out + t * row_bytes;
        for (uint64_t i = lane; i < nv; i += 32) {
            uint4 v[TOPK];
#pragma unroll
            for (int k = 0; k < TOPK; ++k)
                if (k < topk) v[k] = ld128(rk[k] + i * 16);
            float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
            for (int k = 0; k < TOPK; ++k) {
                if (k >= topk) continue;
                float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                acc8(f, v[k]);
#pragma unroll
                for (int j = 0; j < 8; ++j) a[j] += wk[k] * f[j];
            }
            st128(orow + i * 16, pack8(a));
        }
    }
}

// Pack for the MoE dispatch on the verbs: row (t, k) of x goes to rows[start[ids[t, k]] +
// pos[t, k]], so every expert's rows are contiguous and each (owner, expert) group leaves in ONE
// WRITE.  One warp per token: its row is loaded once (16 B per lane per step) and stored to its
// top-k destinations.
template <int TOPK>
__global__ void __launch_bounds__(512) pack_rows_kernel(uint8_t *rows, const uint8_t *x, uint64_t ntok, int topk,
                                                        uint64_t row_bytes, const int32_t *ids, const int32_t *pos,
                                                        const int64_t *start) {
    const int lane = threadIdx.x & 31;
    const uint64_t warp = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = (uint64_t(gridDim.x) * blockDim.x) >> 5;
    const uint64_t nv = row_bytes / 16;
    for (uint64_t t = warp; t < ntok; t += nwarps) {
        uint8_t *dk[TOPK];
#pragma unroll
        for (int k = 0; k < TOPK; ++k) {
            dk[k] = nullptr;
            if (k < topk) {
                const uint64_t r = t * uint64_t(topk) + uint64_t(k);
                dk[k] = rows + (uint64_t(__ldg(start + __ldg(ids + r))) + uint64_t(__ldg(pos + r))) * row_bytes;
            }
        }
        const uint8_t *xr = x + t * row_bytes;
        for (uint64_t i = lane; i < nv; i += 32) {
            const uint4 v = ld128(xr + i * 16);
#pragma unroll
            for (int k = 0; k < TOPK; ++k)
                if (k < topk) st128(dk[k] + i * 16, v);
        }
    }
}

// Counts exchange: this rank's per-expert counts stored into every rank's table
// (table[rank * nexp + e], int32, at byte `table_off` of each buffer), then the end barrier.
__global__ void counts_exchange_kernel(PeerSet ps, const int32_t *counts, int nexp, uint64_t table_off,
                                       uint64_t epoch, uint64_t max_ns) {
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < nexp; e += gridDim.x * blockDim.x) {
        const int32_t c = counts[e];
        for (int q = 0; q < ps.n; ++q) {
            int32_t *t = reinterpret_cast<int32_t *>(reinterpret_cast<uint8_t *>(ps.buf[q]) + table_off);
            t[ps.rank * nexp + e] = c;
        }
    }
    end_barrier(ps, epoch, kSlotCounts, max_ns);
}

// Layout (one block): expert e's group in its owner's receive area starts after the groups of
// the owner's lower experts; this rank's rows for e follow the rows of the lower ranks.
__global__ void layout_kernel(PeerSet ps, int nexp, int exp_per_rank, uint64_t table_off, int64_t *gbase,
                              int64_t *recv_used) {
    const int32_t *t =
        reinterpret_cast<const int32_t *>(reinterpret_cast<const uint8_t *>(ps.buf[ps.rank]) + table_off);
    if (threadIdx.x != 0) return;
    int64_t group = 0;
    for (int e = 0; e < nexp; ++e) {
        if (e % exp_per_rank == 0) group = 0;
        int64_t lower = 0, total = 0;
        for (int q = 0; q < ps.n; ++q) {
            const int64_t c = t[q * nexp + e];
            if (q < ps.rank) lower += c;
            total += c;
        }
        gbase[e] = group + lower;
        group += total;
        if (e / exp_per_rank == ps.rank) *recv_used = group;
    }
}

}  // namespace

int launch_layout(const PeerSet &ps, const int32_t *counts, int nexp, int exp_per_rank, uint64_t table_off,
                  int64_t *gbase, int64_t *recv_used, uint64_t epoch, uint64_t max_ns, cudaStream_t s) {
    counts_exchange_kernel<<<1, 256, 0, s>>>(ps, counts, nexp, table_off, epoch, max_ns);
    layout_kernel<<<1, 32, 0, s>>>(ps, nexp, exp_per_rank, table_off, gbase, recv_used);
    return int(cudaGetLastError());
}

int grid_for(int device) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return sms;
}

int launch_allreduce_bf16(const PeerSet &ps, uint64_t offset, uint64_t count, uint64_t epoch, int ctas,
                          uint64_t max_ns, cudaStream_t s) {
    if (count % 8 != 0 || offset % 16 != 0) return int(cudaErrorInvalidValue);
    const uint64_t nvec = count / 8;
    switch (ps.n) {
    case 1: allreduce_kernel<1><<<ctas, 512, 0, s>>>(ps, offset, nvec, epoch, max_ns); break;
    case 2: allreduce_kernel<2><<<ctas, 512, 0, s>>>(ps, offset, nvec, epoch, max_ns); break;
    case 3: allreduce_kernel<3><<<ctas, 512, 0, s>>>(ps, offset, nvec, epoch, max_ns); break;
    case 4: allreduce_kernel<4><<<ctas, 512, 0, s>>>(ps, offset, nvec, epoch, max_ns); break;
    case 5: allreduce_kernel<5><<<ctas, 512, 0, s>>>(ps, offset, nvec, epoch, max_ns); break;
    case 6: allreduce_kernel<6><<<ctas, 512, 0, s>>>(ps, offset, nvec, epoch, max_ns); break;
    case 7: allreduce_kernel<7><<<ctas, 512, 0, s>>>(ps, offset, nvec, epoch, max_ns); break;
    default: allreduce_kernel<8><<<ctas, 512, 0, s>>>(ps, offset, nvec, epoch, max_ns); break;
    }
    return int(cudaGetLastError());
}

int launch_allreduce_bf16_nvls(const PeerSet &ps, void *mc, uint64_t offset, uint64_t count, uint64_t epoch,
                               int ctas, uint64_t max_ns, cudaStream_t s) {
    if (mc == nullptr || count % 8 != 0 || offset % 16 != 0) return int(cudaErrorInvalidValue);
    // Four 16-byte vectors in flight per thread, one CTA per SM: the fastest of the measured
    // settings on 8 B200, 1 GiB (unroll 4: 2.27 ms at 148 CTAs, 3.26 ms at 296; unroll 8:
    // 2.46 ms at 148, 2.98 ms at 296).
    allreduce_nvls_kernel<4><<<ctas, 512, 0, s>>>(ps, static_cast<uint8_t *>(mc) + offset, count / 8, epoch, max_ns);
    return int(cudaGetLastError());
}

int collective_kernels(const KernelRef **out) {
    static const KernelRef refs[] = {
        {"allreduce_kernel<8>", reinterpret_cast<const void *>(&allreduce_kernel<8>), 512},
        {"allreduce_kernel<2>", reinterpret_cast<const void *>(&allreduce_kernel<2>), 512},
        {"allreduce_nvls_kernel<4>", reinterpret_cast<const void *>(&allreduce_nvls_kernel<4>), 512},
        {"route_hist_kernel", reinterpret_cast<const void *>(&route_hist_kernel), 256},
        {"route_scan_kernel", reinterpret_cast<const void *>(&route_scan_kernel), 128},
        {"route_place_kernel", reinterpret_cast<const void *>(&route_place_kernel), 256},
        {"counts_exchange_kernel", reinterpret_cast<const void *>(&counts_exchange_kernel), 256},
        {"layout_kernel", reinterpret_cast<const void *>(&layout_kernel), 32},
        {"dispatch_kernel", reinterpret_cast<const void *>(&dispatch_kernel), 512},
        {"combine_kernel<8>", reinterpret_cast<const void *>(&combine_kernel<8>), 512},
        {"weighted_rows_kernel<8>", reinterpret_cast<const void *>(&weighted_rows_kernel<8>), 512},
        {"pack_rows_kernel<8>", reinterpret_cast<const void *>(&pack_rows_kernel<8>), 512},
    };
    *out = refs;
    return int(sizeof(refs) / sizeof(refs[0]));
}

size_t route_scratch_bytes(uint64_t rows, int nexp) {
    const uint64_t nblocks = (rows + kRouteRowsPerBlock - 1) / kRouteRowsPerBlock;
    return size_t(nblocks) * size_t(nexp) * sizeof(uint32_t);
}

int launch_route(const int32_t *idx, uint64_t rows, int nexp, int32_t *counts, int32_t *pos, uint32_t *scratch,
                 cudaStream_t s) {
    if (nexp <= 0 || nexp > kRouteMaxExperts) return int(cudaErrorInvalidValue);
    const int nblocks = int((rows + kRouteRowsPerBlock - 1) / kRouteRowsPerBlock);
    const size_t sh = size_t(nexp) * sizeof(uint32_t);
    if (nblocks > 0) route_hist_kernel<<<nblocks, 256, sh, s>>>(idx, rows, nexp, scratch);
    route_scan_kernel<<<(nexp + 127) / 128, 128, 0, s>>>(scratch, nblocks, nexp, counts);
    if (nblocks > 0) route_place_kernel<<<nblocks, 256, sh, s>>>(idx, rows, nexp, scratch, pos);
    return int(cudaGetLastError());
}

int launch_dispatch(const PeerSet &ps, const void *x, uint64_t row_bytes, const int32_t *idx, const int32_t *pos,
                    const int64_t *gbase, uint64_t ntok, int topk, int exp_per_rank, uint64_t recv_off,
                    uint64_t recv_rows, uint64_t epoch, int ctas, uint64_t max_ns, cudaStream_t s) {
    if (row_bytes % 16 != 0) return int(cudaErrorInvalidValue);
    dispatch_kernel<<<ctas, 512, 0, s>>>(ps, static_cast<const uint8_t *>(x), row_bytes, idx, pos, gbase,
                                         ntok * uint64_t(topk), topk, exp_per_rank, recv_off, recv_rows, epoch,
                                         max_ns);
    return int(cudaGetLastError());
}

int launch_combine(const PeerSet &ps, void *out, uint64_t row_bytes, const int32_t *idx, const int32_t *pos,
                   const int64_t *gbase, const float *w, uint64_t ntok, int topk, int exp_per_rank,
                   uint64_t recv_off, uint64_t recv_rows, uint64_t epoch, int ctas, uint64_t max_ns,
                   cudaStream_t s) {
    if (row_bytes % 16 != 0) return int(cudaErrorInvalidValue);
    if (topk <= 0 || topk > 16) return int(cudaErrorInvalidValue);
    uint8_t *o = static_cast<uint8_t *>(out);
#define UGDR_COMBINE(K)                                                                                  \
    combine_kernel<K><<<ctas, 512, 0, s>>>(ps, o, row_bytes, idx, pos, gbase, w, ntok, topk, exp_per_rank, \
                                           recv_off, recv_rows, epoch, max_ns)
    if (topk <= 2)
        UGDR_COMBINE(2);
    else if (topk <= 4)
        UGDR_COMBINE(4);
    else if (topk <= 8)
        UGDR_COMBINE(8);
    else
        UGDR_COMBINE(16);
#undef UGDR_COMBINE
    return int(cudaGetLastError());
}

int launch_weighted_rows(void *out, const void *rows, const float *w, uint64_t ntok, int topk, uint64_t row_bytes,
                         int ctas, cudaStream_t s, const int32_t *ids, const int32_t *pos, const int64_t *start) {
    if (row_bytes % 16 != 0 || topk <= 0 || topk > 16) return int(cudaErrorInvalidValue);
    uint8_t *o = static_cast<uint8_t *>(out);
    const uint8_t *r = static_cast<const uint8_t *>(rows);
    if (topk <= 2)
        weighted_rows_kernel<2><<<ctas, 512, 0, s>>>(o, r, w, ntok, topk, row_bytes, ids, pos, start);
    else if (topk <= 4)
        weighted_rows_kernel<4><<<ctas, 512, 0, s>>>(o, r, w, ntok, topk, row_bytes, ids, pos, start);
    else if (topk <= 8)
        weighted_rows_kernel<8><<<ctas, 512, 0, s>>>(o, r, w, ntok, topk, row_bytes, ids, pos, start);
    else
        weighted_rows_kernel<16><<<ctas, 512, 0, s>>>(o, r, w, ntok, topk, row_bytes, ids, pos, start);
    return int(cudaGetLastError());
}

int launch_pack_rows(void *rows, const void *x, uint64_t ntok, int topk, uint64_t row_bytes, const int32_t *ids,
                     const int32_t *pos, const int64_t *start, int ctas, cudaStream_t s) {
    if (row_bytes % 16 != 0 || topk <= 0 || topk > 16) return int(cudaErrorInvalidValue);
    uint8_t *o = static_cast<uint8_t *>(rows);
    const uint8_t *r = static_cast<const uint8_t *>(x);
    if (topk <= 2)
        pack_rows_kernel<2><<<ctas, 512, 0, s>>>(o, r, ntok, topk, row_bytes, ids, pos, start);
    else if (topk <= 4)
        pack_rows_kernel<4><<<ctas, 512, 0, s>>>(o, r, ntok, topk, row_bytes, ids, pos, start);
    else if (topk <= 8)
        pack_rows_kernel<8><<<ctas, 512, 0, s>>>(o, r, ntok, topk, row_bytes, ids, pos, start);
    else
        pack_rows_kernel<16><<<ctas, 512, 0, s>>>(o, r, ntok, topk, row_bytes, ids, pos, start);
    return int(cudaGetLastError());
}

}  // namespace ugdr::coll
