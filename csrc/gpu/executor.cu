// Persistent sm_100a executor: polls QP send rings, executes RDMA WRITE / WRITE_WITH_IMM /
// READ / 8-byte atomics with direct loads and stores to peer (NVLink) or local memory, and
// writes completions straight into the clients' CQ rings.
//
// Parity: replaces the reference's LoopWorker + LocalTransport + PersistentCudaCopyBackend +
// warp_specialized_pipeline_kernel chain (src/worker/worker.cpp:63-509,
// src/gpu/persistent_copy_backend.cu:429-692, src/gpu/persistent_copy.cu:893-1079).  The
// reference's kernel is one CTA fed 8 KiB copy tasks by a host thread; here the host is off the
// data path entirely:
//
//  * Ownership.  QP slot q belongs to exactly one warp of the grid (CTA q % grid, warp
//    (q / grid) % warps), so each QP's WRs are fetched, validated and retired in posting order by
//    one warp, and QPs spread over all SMs.
//  * Issue.  The owner warp reads the WQE (host-mapped ring) lane-parallel into shared memory,
//    resolves every SGE's lkey and the rkey against the device MR table, and either copies the
//    payload itself (<= 4 KiB, atomics) or publishes it as a job whose fixed-size chunks any
//    warp on the GPU may claim (CAS on a generation-tagged counter), so a single large WR
//    spreads over every SM.
//  * Retire.  When all chunks of the oldest in-flight WR are done the owner produces the receive
//    CQE (WRITE_WITH_IMM), the send CQE (signaled or error), and advances the ring head.  CQs
//    are multi-producer (several warps, several GPUs): slots are reserved by CAS against the
//    consumer cursor and published strictly in order.
//  * Bounded waits.  Every spin carries a %globaltimer deadline; on expiry the kernel records
//    the reason in DevStats::error_code and every warp exits.  There is no __trap, assert or
//    unbounded loop.  The kernel also exits after `idle_exit_ns` without work, on a host stop
//    flag, or (drain mode) once `expected` WRs retired; in-flight state lives in device memory
//    so a relaunch resumes where the previous launch stopped.
#include "gpu/device_abi.hpp"
#include "gpu/executor.hpp"
#include "ugdr/api.hpp"

#include <cuda_runtime.h>
#include <stdint.h>

namespace ugdr::gpu {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr uint32_t kWqeBytesMax = 576;  // roundup64(40 + 16 * 32)
constexpr uint32_t kChunkMin = 16384;
constexpr uint32_t kChunkMax = 262144;

// ---- memory-model helpers --------------------------------------------------------------------

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
__device__ __forceinline__ uint32_t ld_acq_sys32(const void *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_rel_sys(void *p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_vol(const void *p) {
    uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_vol32(const void *p) {
    uint32_t v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint4 ld_vol128(const void *p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ void st_vol128(void *p, uint4 v) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ uint4 ld128(const void *p) {
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ void st128(void *p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

template <typename T> __device__ __forceinline__ T bcast(T v) {
    return __shfl_sync(0xffffffffu, v, 0);
}
__device__ __forceinline__ uint64_t bcast64(uint64_t v) {
    return (uint64_t(__shfl_sync(0xffffffffu, uint32_t(v >> 32), 0)) << 32) |
           __shfl_sync(0xffffffffu, uint32_t(v), 0);
}

// ---- warp copy core ----------------------------------------------------------------------------
// Copies n bytes, never touching bytes outside [dst, dst + n) / [src, src + n).  16-byte vector
// body when both pointers share their offset mod 16 (8 vectors in flight per lane), 4-byte body
// when they share it mod 4, bytes otherwise.

__device__ void warp_copy(uint8_t *dst, const uint8_t *src, uint64_t n, int lane) {
    if (n == 0) return;
    const uintptr_t d = reinterpret_cast<uintptr_t>(dst), s = reinterpret_cast<uintptr_t>(src);
    if (((d ^ s) & 15) == 0 && n >= 64) {
        uint64_t head = (16 - (d & 15)) & 15;
        if (head > n) head = n;
        if (uint64_t(lane) < head) dst[lane] = src[lane];
        dst += head;
        src += head;
        n -= head;
        const uint64_t nvec = n >> 4;
        uint4 *dv = reinterpret_cast<uint4 *>(dst);
        const uint4 *sv = reinterpret_cast<const uint4 *>(src);
        constexpr int U = 8;
        uint64_t i = lane;
        for (; i + (U - 1) * 32 < nvec; i += U * 32) {
            uint4 r[U];
#pragma unroll
            for (int u = 0; u < U; ++u) r[u] = ld128(sv + i + u * 32);
#pragma unroll
            for (int u = 0; u < U; ++u) st128(dv + i + u * 32, r[u]);
        }
        for (; i < nvec; i += 32) st128(dv + i, ld128(sv + i));
        const uint64_t done = nvec << 4;
        const uint64_t tail = n - done;
        if (uint64_t(lane) < tail) dst[done + lane] = src[done + lane];
        return;
    }
    if (((d ^ s) & 3) == 0 && n >= 16) {
        uint64_t head = (4 - (d & 3)) & 3;
        if (head > n) head = n;
        if (uint64_t(lane) < head) dst[lane] = src[lane];
        dst += head;
        src += head;
        n -= head;
        const uint64_t nw = n >> 2;
        uint32_t *dw = reinterpret_cast<uint32_t *>(dst);
        const uint32_t *sw = reinterpret_cast<const uint32_t *>(src);
        for (uint64_t i = lane; i < nw; i += 32) dw[i] = sw[i];
        const uint64_t done = nw << 2;
        if (uint64_t(lane) < n - done) dst[done + lane] = src[done + lane];
        return;
    }
    for (uint64_t i = lane; i < n; i += 32) dst[i] = src[i];
}

// Copy stream bytes [off, off + len) of a WR: local segments <-> contiguous remote range.
__device__ void copy_stream(const WrRec *rec, uint32_t nseg, uint64_t remote, bool to_remote,
                            uint64_t off, uint64_t len, int lane) {
    uint64_t seg_start = 0;
    for (uint32_t i = 0; i < nseg && len > 0; ++i) {
        const uint64_t sl = __ldcg(reinterpret_cast<const unsigned long long *>(&rec->seg[i].length));
        if (off < seg_start + sl) {
            const uint64_t in = off - seg_start;
            uint64_t take = sl - in;
            if (take > len) take = len;
            uint8_t *local = reinterpret_cast<uint8_t *>(
                                 __ldcg(reinterpret_cast<const unsigned long long *>(&rec->seg[i].local))) +
                             in;
            uint8_t *rem = reinterpret_cast<uint8_t *>(remote) + off;
            if (to_remote)
                warp_copy(rem, local, take, lane);
            else
                warp_copy(local, rem, take, lane);
            off += take;
            len -= take;
        }
        seg_start += sl;
    }
}

// ---- per-launch warp context -------------------------------------------------------------------

struct Warp {
    const ExecParams *p;
    int lane;
    uint32_t wi;    // warp index inside the CTA
    uint32_t gwarp; // global warp index
    uint32_t rot;   // job-slot rotation seed
    bool abort;
    // Private counters, folded into DevStats now and then (hot shared counters would serialise
    // every warp of the grid on one L2 line).
    uint64_t n_chunks, n_miss, bytes, busy;
};

__device__ void record_error(Warp &w, uint32_t code) {
    if (w.lane == 0) {
        atomicCAS(&w.p->stats->error_code, 0u, code);
        atomicAdd(&w.p->stats->wait_timeouts, 1ull);
        atomicExch(&w.p->stats->exiting, 1u);
    }
    w.abort = true;
}

// Bounded wait (lane 0) until *p == want; returns false on timeout.
__device__ bool wait_eq_sys(const unsigned long long *p, uint64_t want, uint64_t max_ns) {
    const uint64_t t0 = gtime();
    uint32_t spins = 0;
    while (ld_acq_sys(p) != want) {
        if ((++spins & 63) == 0 && gtime() - t0 > max_ns) return false;
        __nanosleep(32);
    }
    return true;
}

// Multi-producer CQE publish (lane 0 only).  Returns 0 = published, 1 = CQ full (retry later),
// 2 = publish wait timed out.
__device__ int produce_cqe(DevCq *cq, const queue::Cqe &e, uint64_t max_ns) {
    const uint32_t cap = ld_vol32(&cq->cfg.capacity);
    queue::RingHeader *ring = reinterpret_cast<queue::RingHeader *>(ld_vol(&cq->cfg.ring));
    uint8_t *slots = reinterpret_cast<uint8_t *>(ld_vol(&cq->cfg.slots));
    const uint32_t stride = ld_vol32(&cq->cfg.stride);
    uint64_t r;
    for (int attempt = 0;; ++attempt) {
        r = ld_acq_sys(&cq->st.reserve);
        uint64_t head = ld_acq_sys(&cq->st.head_seen);
        if (r - head >= cap) {
            head = ld_acq_sys(&ring->head.value);
            atomicMax_system(&cq->st.head_seen, head);
            if (r - head >= cap) return 1;
        }
        if (atomicCAS_system(&cq->st.reserve, r, r + 1) == r) break;
        if (attempt > 1000) return 1;
    }
    uint8_t *slot = slots + (r % cap) * stride;
    const uint4 *src = reinterpret_cast<const uint4 *>(&e);
    st_vol128(slot, src[0]);
    st_vol128(slot + 16, src[1]);
    if (!wait_eq_sys(&cq->st.published, r, max_ns)) return 2;
    __threadfence_system();
    st_rel_sys(&ring->tail.value, r + 1);
    st_rel_sys(&cq->st.published, r + 1);
    return 0;
}

// Claim the next RQ WR of `qp` (lane 0).  Returns false when the RQ is empty.
__device__ bool claim_rq(DevQp *qp, uint64_t *claim, uint64_t *wr_id) {
    queue::RingHeader *rq = reinterpret_cast<queue::RingHeader *>(ld_vol(&qp->cfg.rq));
    for (int attempt = 0; attempt < 64; ++attempt) {
        const uint64_t c = ld_acq_sys(&qp->st.rq_claim);
        const uint64_t tail = ld_acq_sys(&rq->tail.value);
        if (c >= tail) return false;
        if (atomicCAS_system(&qp->st.rq_claim, c, c + 1) == c) {
            const uint8_t *slots = reinterpret_cast<const uint8_t *>(ld_vol(&qp->cfg.rq_slots));
            const uint32_t cap = ld_vol32(&qp->cfg.rq_cap), stride = ld_vol32(&qp->cfg.rq_stride);
            *wr_id = ld_vol(slots + (c % cap) * stride);
            *claim = c;
            return true;
        }
    }
    return false;
}

// Publish RQ consumption in order (lane 0).
__device__ bool release_rq(DevQp *qp, uint64_t claim, uint64_t max_ns) {
    if (!wait_eq_sys(&qp->st.rq_released, claim, max_ns)) return false;
    queue::RingHeader *rq = reinterpret_cast<queue::RingHeader *>(ld_vol(&qp->cfg.rq));
    st_rel_sys(&rq->head.value, claim + 1);
    st_rel_sys(&qp->st.rq_released, claim + 1);
    return true;
}

__device__ __forceinline__ uint32_t wc_op(uint32_t op) {
    switch (op) {
    case UGDR_WR_RDMA_READ: return UGDR_WC_RDMA_READ;
    case UGDR_WR_ATOMIC_CMP_AND_SWP: return UGDR_WC_COMP_SWAP;
    case UGDR_WR_ATOMIC_FETCH_AND_ADD: return UGDR_WC_FETCH_ADD;
    default: return UGDR_WC_RDMA_WRITE;
    }
}
__device__ __forceinline__ bool is_atomic(uint32_t op) {
    return op == UGDR_WR_ATOMIC_CMP_AND_SWP || op == UGDR_WR_ATOMIC_FETCH_AND_ADD;
}
__device__ __forceinline__ uint32_t remote_need(uint32_t op) {
    if (op == UGDR_WR_RDMA_READ) return UGDR_ACCESS_REMOTE_READ;
    if (is_atomic(op)) return UGDR_ACCESS_REMOTE_ATOMIC;
    return UGDR_ACCESS_REMOTE_WRITE;
}
__device__ uint64_t rnr_ns(uint32_t code) {
    constexpr uint32_t t[32] = {65536, 1,    2,    3,    4,    6,    8,     12,    16,   24,   32,
                            48,    64,   96,   128,  192,  256,  384,   512,   768,  1024, 1536,
                            2048,  3072, 4096, 6144, 8192, 12288, 16384, 24576, 32768, 49152};
    return uint64_t(t[code & 31]) * 10000ull;
}

// ---- jobs ------------------------------------------------------------------------------------

// Publish `rec` as a chunked job (lane 0).  Returns false when no job slot is free.
__device__ bool publish_job(JobRing *jr, uint32_t *bitmap, WrRec *rec, uint32_t nchunks,
                            uint32_t chunk_bytes, uint32_t seed) {
    for (uint32_t k = 0; k < 64; ++k) {
        const uint32_t s = (seed * 37u + k * 97u) % kJobSlots;
        Job *j = &jr->slots[s];
        // Slot free <=> seq even; taking it makes seq odd.  gen = (seq + 1) / 2 is new each time.
        const unsigned long long seq = ld_vol(&j->seq);
        if ((seq & 1ull) != 0) continue;
        if (atomicCAS(&j->seq, seq, seq + 1) != seq) continue;
        j->rec = rec;
        j->nchunks = nchunks;
        j->chunk_bytes = chunk_bytes;
        const unsigned long long gen = (seq + 1) >> 1;
        __threadfence();
        atomicExch(&j->ctl, (gen << 32) | 0ull);
        __threadfence();
        atomicOr(&bitmap[s >> 5], 1u << (s & 31));
        return true;
    }
    return false;
}

struct Claim {
    WrRec *rec;
    Job *job;
    uint32_t chunk, cb, n;
};

// Claim one chunk from any active job (warp-wide): a fetch-and-add on the job's counter, which
// always yields a unique index (no CAS retry storms when thousands of warps contend).
//  * The fields are read before the add; if the add returns the same generation, no recycle
//    happened in between, so the fields belong to it (a slot is recycled only after all of its
//    chunks are done, which cannot be while our index is below nchunks).
//  * If the add lands in a newer generation, the index belongs to that job: re-read its fields
//    (stable for the same reason) and run it, so no index is ever lost.
// `mirror` is the CTA's shared copy of the active-job bitmap (refreshed by the CTA leader).
__device__ bool claim_chunk(Warp &w, JobRing *jr, uint32_t *bitmap, const volatile uint32_t *mirror,
                            Claim *out) {
    const uint32_t word = mirror[w.lane];
    const uint32_t nonzero = __ballot_sync(0xffffffffu, word != 0);
    if (nonzero == 0) return false;
    int got = 0;
    Claim cl{};
    if (w.lane == 0) {
        // Rotate the starting word / bit per warp so warps spread over active jobs.
        const uint32_t rotw = w.rot & 31;
        const uint32_t nz = (nonzero >> rotw) | (nonzero << ((32 - rotw) & 31));
        const uint32_t wsel = (rotw + __ffs(nz) - 1) & 31;
        const uint32_t bits = mirror[wsel];
        if (bits != 0) {
            const uint32_t rb = (w.rot >> 5) & 31;
            const uint32_t rotated = (bits >> rb) | (bits << ((32 - rb) & 31));
            const uint32_t b = (rb + __ffs(rotated) - 1) & 31;
            Job *j = &jr->slots[wsel * 32 + b];
            const unsigned long long v0 = ld_vol(&j->ctl);
            const uint4 f = ld_vol128(&j->rec);  // rec (x,y), nchunks (z), chunk_bytes (w)
            if (uint32_t(v0) < f.z) {
                const unsigned long long v = atomicAdd(&j->ctl, 1ull);
                uint4 g = f;
                if ((v >> 32) != (v0 >> 32)) g = ld_vol128(&j->rec);  // newer generation
                const uint32_t c = uint32_t(v);
                if (c < g.z) {
                    got = 1;
                    cl.rec = reinterpret_cast<WrRec *>((uint64_t(g.y) << 32) | g.x);
                    cl.job = j;
                    cl.chunk = c;
                    cl.n = g.z;
                    cl.cb = g.w;
                    if (c + 1 == g.z) atomicAnd(&bitmap[wsel], ~(1u << b));  // all handed out
                }
            }
        }
        w.rot = w.rot * 1664525u + 1013904223u;
    }
    w.rot = __shfl_sync(0xffffffffu, w.rot, 0);
    got = __shfl_sync(0xffffffffu, got, 0);
    if (!got) {
        w.n_miss += 1;
        return false;
    }
    out->rec = reinterpret_cast<WrRec *>(bcast64(reinterpret_cast<uint64_t>(cl.rec)));
    out->job = reinterpret_cast<Job *>(bcast64(reinterpret_cast<uint64_t>(cl.job)));
    out->chunk = bcast(cl.chunk);
    out->cb = bcast(cl.cb);
    out->n = bcast(cl.n);
    return true;
}

__device__ void run_chunk(Warp &w, const Claim &cl) {
    WrRec *rec = cl.rec;
    const uint64_t total = ld_vol(&rec->total);
    const uint64_t off = uint64_t(cl.chunk) * cl.cb;
    uint64_t len = total - off;
    if (len > cl.cb) len = cl.cb;
    const uint32_t op = ld_vol32(&rec->opcode);
    const uint32_t nseg = ld_vol32(&rec->nseg);
    const uint64_t remote = ld_vol(&rec->remote);
    const uint64_t t0 = gtime();
    copy_stream(rec, nseg, remote, op != UGDR_WR_RDMA_READ, off, len, w.lane);
    __syncwarp();
    if (w.lane == 0) {
        // Device-scope release is enough here: the owner warp acquires chunks_done and issues
        // the system-scope fence before it publishes the CQE, and causality is transitive.
        __threadfence();
        const uint32_t done = atomicAdd(&rec->chunks_done, 1u) + 1;
        if (done == cl.n) atomicAdd(&cl.job->seq, 1ull);  // every chunk done: free the slot
    }
    w.n_chunks += 1;
    w.bytes += len;
    w.busy += gtime() - t0;
}

// Fold the warp's private counters into DevStats (lane 0).
__device__ void flush_counters(Warp &w) {
    if (w.lane == 0) {
        if (w.n_chunks) atomicAdd(&w.p->stats->chunks_run, (unsigned long long)w.n_chunks);
        if (w.n_miss) atomicAdd(&w.p->stats->claim_misses, (unsigned long long)w.n_miss);
        if (w.bytes) atomicAdd(&w.p->stats->bytes_moved, (unsigned long long)w.bytes);
        if (w.busy) atomicAdd(&w.p->stats->busy_ns, (unsigned long long)w.busy);
    }
    w.n_chunks = w.n_miss = w.bytes = w.busy = 0;
}

// ---- per-QP service ----------------------------------------------------------------------------

struct WqeView {
    queue::SendWqe h;
    uint64_t compare_add;
};

// Validate and stage one WQE (already in shared memory `wqe`) into `rec`.  Warp-wide.
__device__ void stage_wr(Warp &w, DevQp *qp, const uint8_t *wqe, WrRec *rec, uint32_t *status_out,
                         uint64_t *total_out, uint64_t *remote_out) {
    const queue::SendWqe *h = reinterpret_cast<const queue::SendWqe *>(wqe);
    const uint32_t op = h->opcode;
    const uint32_t nsge = h->sge_count;
    const uint32_t max_sge = ld_vol32(&qp->cfg.max_send_sge);
    const uint32_t pd = ld_vol32(&qp->cfg.pd_num);
    uint32_t status = UGDR_WC_SUCCESS;
    const bool op_ok = op == UGDR_WR_RDMA_WRITE || op == UGDR_WR_RDMA_WRITE_WITH_IMM ||
                       op == UGDR_WR_RDMA_READ || is_atomic(op);
    if (!op_ok || nsge > max_sge || nsge > kMaxSge || (is_atomic(op) && nsge != 1))
        status = UGDR_WC_LOC_QP_OP_ERR;
    // Lane i resolves SGE i.
    uint64_t len = 0, local = 0;
    bool bad = false;
    if (status == UGDR_WC_SUCCESS && uint32_t(w.lane) < nsge) {
        const queue::Sge *sg =
            reinterpret_cast<const queue::Sge *>(wqe + queue::kSendSgeOffset) + w.lane;
        len = sg->length;
        if (len != 0) {
            const DevMr *m = &w.p->mrs[(sg->lkey >> 1) & (kMaxMrs - 1)];
            const uint32_t valid = ld_vol32(&m->valid);
            const uint32_t lkey = ld_vol32(&m->lkey);
            const uint64_t cb = ld_vol(&m->client_base), ml = ld_vol(&m->length);
            const uint64_t base = ld_vol(&m->base);
            const uint32_t acc = ld_vol32(&m->access), mpd = ld_vol32(&m->pd_num);
            const bool need_write = op == UGDR_WR_RDMA_READ || is_atomic(op);
            if (!valid || lkey != sg->lkey || mpd != pd || base == 0 || sg->address < cb ||
                len > ml || sg->address - cb > ml - len ||
                (need_write && (acc & UGDR_ACCESS_LOCAL_WRITE) == 0)) {
                bad = true;
            } else {
                local = base + (sg->address - cb);
            }
        }
    }
    const bool any_bad = __any_sync(0xffffffffu, bad);
    uint64_t total = len;
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (status == UGDR_WC_SUCCESS && any_bad) status = UGDR_WC_LOC_PROT_ERR;
    if (status == UGDR_WC_SUCCESS && total > 0x80000000ull) status = UGDR_WC_LOC_LEN_ERR;
    if (status == UGDR_WC_SUCCESS && is_atomic(op) && total != 8) status = UGDR_WC_LOC_LEN_ERR;

    // Compact the non-empty segments: lane i keeps slot = prefix count of non-empty lanes.
    const bool keep = uint32_t(w.lane) < nsge && len != 0;
    const uint32_t keep_mask = __ballot_sync(0xffffffffu, keep);
    if (keep && status == UGDR_WC_SUCCESS) {
        const uint32_t idx = __popc(keep_mask & ((1u << w.lane) - 1));
        rec->seg[idx].local = local;
        rec->seg[idx].length = len;
    }

    // Remote side (uniform).
    uint64_t remote = 0;
    if (status == UGDR_WC_SUCCESS) {
        DevQp *peer = reinterpret_cast<DevQp *>(ld_vol(&qp->cfg.peer));
        const uint32_t lost = ld_vol32(&qp->cfg.peer_lost);
        uint32_t pstate = 0, perr = 0;
        if (peer != nullptr) {
            pstate = ld_acq_sys32(&peer->cfg.state);
            perr = ld_acq_sys32(&peer->st.err);
        }
        if (peer == nullptr || lost || pstate == UGDR_QPS_RESET || !ld_acq_sys32(&peer->cfg.active)) {
            status = UGDR_WC_RETRY_EXC_ERR;
        } else if (pstate == UGDR_QPS_ERR || perr) {
            status = UGDR_WC_REM_OP_ERR;
        } else {
            const uint32_t need = remote_need(op);
            const uint32_t pacc = ld_acq_sys32(&peer->cfg.access);
            const uint32_t ppd = ld_acq_sys32(&peer->cfg.pd_num);
            const uint64_t rlen = is_atomic(op) ? 8 : total;
            if ((pacc & need) == 0) {
                status = UGDR_WC_REM_ACCESS_ERR;
            } else if (rlen != 0) {
                const DevMr *m = &w.p->mrs[(h->rkey >> 1) & (kMaxMrs - 1)];
                const uint32_t valid = ld_vol32(&m->valid), rkey = ld_vol32(&m->rkey);
                const uint64_t cb = ld_vol(&m->client_base), ml = ld_vol(&m->length);
                const uint64_t base = ld_vol(&m->base);
                const uint32_t acc = ld_vol32(&m->access), mpd = ld_vol32(&m->pd_num);
                const uint64_t ra = h->remote_address;
                if (!valid || rkey != h->rkey || mpd != ppd || base == 0 || (acc & need) == 0 ||
                    ra < cb || rlen > ml || ra - cb > ml - rlen)
                    status = UGDR_WC_REM_ACCESS_ERR;
                else
                    remote = base + (ra - cb);
                if (status == UGDR_WC_SUCCESS && is_atomic(op) && (ra & 7) != 0)
                    status = UGDR_WC_REM_INV_REQ_ERR;
            }
        }
    }
    if (w.lane == 0) {
        rec->wr_id = h->wr_id;
        rec->opcode = op;
        rec->total = total;
        rec->remote = remote;
        rec->status = status;
        rec->imm = h->immediate_data;
        rec->nseg = __popc(keep_mask);
        rec->recv_cqe_done = 0;
        rec->chunks_done = 0;
        rec->nchunks = 0;
    }
    __syncwarp();
    *status_out = status;
    *total_out = total;
    *remote_out = remote;
}

// Execute an inline WR (small payload or atomic) with the owner warp.
__device__ void run_inline(Warp &w, WrRec *rec, const uint8_t *wqe, uint32_t op, uint64_t total,
                           uint64_t remote) {
    const uint32_t nseg = ld_vol32(&rec->nseg);
    if (is_atomic(op)) {
        if (w.lane == 0) {
            const queue::SendWqe *h = reinterpret_cast<const queue::SendWqe *>(wqe);
            uint64_t cmp;
            memcpy(&cmp, wqe + queue::kAtomicCompareOffset, 8);
            const uint64_t swap = (uint64_t(h->reserved) << 32) | h->immediate_data;
            unsigned long long *t = reinterpret_cast<unsigned long long *>(remote);
            unsigned long long old;
            if (op == UGDR_WR_ATOMIC_FETCH_AND_ADD)
                old = atomicAdd_system(t, (unsigned long long)cmp);
            else
                old = atomicCAS_system(t, (unsigned long long)cmp, (unsigned long long)swap);
            uint8_t *dst = reinterpret_cast<uint8_t *>(rec->seg[0].local);
            memcpy(dst, &old, 8);
            __threadfence_system();
            atomicAdd(&w.p->stats->bytes_moved, 8ull);
        }
        __syncwarp();
        return;
    }
    copy_stream(rec, nseg, remote, op != UGDR_WR_RDMA_READ, 0, total, w.lane);
    __syncwarp();
    if (w.lane == 0) {
        __threadfence_system();
        atomicAdd(&w.p->stats->bytes_moved, (unsigned long long)total);
    }
}

// Service one QP: retire finished WRs, then issue new ones.  Warp-wide; returns work done.
__device__ uint32_t service_qp(Warp &w, DevQp *qp, uint8_t *wqe_smem, JobRing *jr, uint32_t *bitmap,
                               uint32_t nwarps) {
    if (!ld_vol32(&qp->cfg.active)) return 0;
    const uint64_t max_ns = w.p->max_wait_ns;
    queue::RingHeader *sq = reinterpret_cast<queue::RingHeader *>(ld_vol(&qp->cfg.sq));
    const uint8_t *sq_slots = reinterpret_cast<const uint8_t *>(ld_vol(&qp->cfg.sq_slots));
    const uint32_t sq_cap = ld_vol32(&qp->cfg.sq_cap), sq_stride = ld_vol32(&qp->cfg.sq_stride);
    const uint32_t qpn = ld_vol32(&qp->cfg.qpn);
    uint32_t work = 0;

    // Retire in order.
    for (;;) {
        int verdict = 0;  // 0 stop, 1 retired one
        if (w.lane == 0) {
            const uint64_t head = qp->st.sq_head, issue = qp->st.sq_issue;
            if (head < issue) {
                WrRec *rec = &qp->st.win[head % kWindow];
                const uint32_t n = ld_vol32(&rec->nchunks);
                const uint32_t done = atomicAdd(&rec->chunks_done, 0u);
                if (done >= n) {
                    __threadfence();
                    verdict = 1;
                    const uint32_t op = rec->opcode, status = rec->status;
                    if (status == UGDR_WC_SUCCESS && op == UGDR_WR_RDMA_WRITE_WITH_IMM &&
                        !rec->recv_cqe_done) {
                        DevQp *peer = reinterpret_cast<DevQp *>(ld_vol(&qp->cfg.peer));
                        queue::Cqe rc{rec->recv_wr_id, UGDR_WC_SUCCESS, UGDR_WC_RECV_RDMA_WITH_IMM,
                                      uint32_t(rec->total), rec->imm,
                                      peer ? ld_acq_sys32(&peer->cfg.qpn) : 0u, UGDR_WC_WITH_IMM};
                        DevCq *rcq = peer ? reinterpret_cast<DevCq *>(ld_vol(&peer->cfg.recv_cq)) : nullptr;
                        const int prc = rcq ? produce_cqe(rcq, rc, max_ns) : 0;
                        if (prc == 1) {
                            verdict = 0;
                        } else if (prc == 2) {
                            verdict = -1;
                        } else {
                            if (peer && !release_rq(peer, rec->recv_claim, max_ns)) verdict = -2;
                            rec->recv_cqe_done = 1;
                        }
                    }
                    if (verdict == 1 && (rec->signaled || status != UGDR_WC_SUCCESS)) {
                        queue::Cqe c{rec->wr_id, status, wc_op(op),
                                     status == UGDR_WC_SUCCESS ? uint32_t(rec->total) : 0u, 0u, qpn, 0u};
                        DevCq *scq = reinterpret_cast<DevCq *>(ld_vol(&qp->cfg.send_cq));
                        const int prc = produce_cqe(scq, c, max_ns);
                        if (prc == 1) verdict = 0;
                        if (prc == 2) verdict = -1;
                    }
                    if (verdict == 1) {
                        qp->st.sq_head = head + 1;
                        st_rel_sys(&sq->head.value, head + 1);
                        atomicAdd(&w.p->stats->wrs_completed, 1ull);
                        atomicAdd(&w.p->stats->retired, 1ull);
                        atomicMax(&w.p->stats->last_end_ns, (unsigned long long)gtime());
                        if (status != UGDR_WC_SUCCESS) {
                            atomicAdd(&w.p->stats->error_completions, 1ull);
                            qp->st.err = 1;
                            st_rel_sys(&sq->meta.reserved[queue::kQpErrorWordIndex], UGDR_QPS_ERR);
                        }
                    }
                }
            }
        }
        verdict = bcast(verdict);
        if (verdict < 0) {
            record_error(w, verdict == -1 ? kErrCqPublishTimeout : kErrRqReleaseTimeout);
            return work;
        }
        if (verdict == 0) break;
        ++work;
    }

    const uint32_t state = ld_vol32(&qp->cfg.state);
    const bool in_error = state == UGDR_QPS_ERR || ld_vol32(&qp->st.err) != 0;
    if (in_error) {
        // Flush once nothing is in flight: every unissued SQ WR and every posted RQ WR.
        int flushed = 0;
        if (w.lane == 0 && qp->st.sq_head == qp->st.sq_issue) {
            DevCq *scq = reinterpret_cast<DevCq *>(ld_vol(&qp->cfg.send_cq));
            DevCq *rcq = reinterpret_cast<DevCq *>(ld_vol(&qp->cfg.recv_cq));
            const uint64_t tail = ld_acq_sys(&sq->tail.value);
            while (qp->st.sq_issue < tail && flushed >= 0) {
                const uint8_t *slot = sq_slots + (qp->st.sq_issue % sq_cap) * sq_stride;
                const uint64_t wr_id = ld_vol(slot);
                const uint32_t op = ld_vol32(slot + 20);
                queue::Cqe c{wr_id, UGDR_WC_WR_FLUSH_ERR, wc_op(op), 0u, 0u, qpn, 0u};
                const int prc = produce_cqe(scq, c, max_ns);
                if (prc == 1) break;
                if (prc == 2) {
                    flushed = -1;
                    break;
                }
                qp->st.sq_issue += 1;
                qp->st.sq_head = qp->st.sq_issue;
                st_rel_sys(&sq->head.value, qp->st.sq_head);
                atomicAdd(&w.p->stats->error_completions, 1ull);
                atomicAdd(&w.p->stats->retired, 1ull);
                ++flushed;
            }
            uint64_t claim = 0, wr_id = 0;
            while (flushed >= 0 && claim_rq(qp, &claim, &wr_id)) {
                queue::Cqe c{wr_id, UGDR_WC_WR_FLUSH_ERR, UGDR_WC_RECV_RDMA_WITH_IMM, 0u, 0u, qpn, 0u};
                // Receive CQ full: the claim stays open and is retried by the next pass.
                int prc;
                const uint64_t t0 = gtime();
                while ((prc = produce_cqe(rcq, c, max_ns)) == 1 && gtime() - t0 < max_ns) __nanosleep(256);
                if (prc != 0 || !release_rq(qp, claim, max_ns)) {
                    flushed = -2;
                    break;
                }
                atomicAdd(&w.p->stats->error_completions, 1ull);
                ++flushed;
            }
        }
        flushed = bcast(flushed);
        if (flushed < 0) record_error(w, flushed == -1 ? kErrCqPublishTimeout : kErrRqReleaseTimeout);
        return work + (flushed > 0 ? flushed : 0);
    }
    if (state != UGDR_QPS_RTS) return work;

    // Issue.
    const uint32_t sig_all = ld_vol32(&qp->cfg.sq_sig_all);
    uint64_t tail = 0;
    if (w.lane == 0) tail = ld_acq_sys(&sq->tail.value);
    tail = bcast64(tail);
    for (;;) {
        const uint64_t head = ld_vol(&qp->st.sq_head), issue = ld_vol(&qp->st.sq_issue);
        if (issue >= tail || issue - head >= kWindow) break;
        // Fetch the WQE lane-parallel (16 B per lane) into shared memory.
        const uint8_t *slot = sq_slots + (issue % sq_cap) * sq_stride;
        for (uint32_t o = w.lane * 16; o < sq_stride && o < kWqeBytesMax; o += 32 * 16)
            *reinterpret_cast<uint4 *>(wqe_smem + o) = ld_vol128(slot + o);
        __syncwarp();
        WrRec *rec = &qp->st.win[issue % kWindow];
        uint32_t status;
        uint64_t total, remote;
        stage_wr(w, qp, wqe_smem, rec, &status, &total, &remote);
        const queue::SendWqe *h = reinterpret_cast<const queue::SendWqe *>(wqe_smem);
        const uint32_t op = h->opcode;
        const bool signaled = sig_all || (h->send_flags & UGDR_SEND_SIGNALED) != 0;

        // Responder RQ for WRITE_WITH_IMM (RNR when empty).
        int rnr = 0;  // 0 go, 1 wait, 2 retry budget exhausted
        if (status == UGDR_WC_SUCCESS && op == UGDR_WR_RDMA_WRITE_WITH_IMM) {
            if (w.lane == 0) {
                DevQp *peer = reinterpret_cast<DevQp *>(ld_vol(&qp->cfg.peer));
                uint64_t claim = 0, wr_id = 0;
                if (claim_rq(peer, &claim, &wr_id)) {
                    rec->recv_claim = claim;
                    rec->recv_wr_id = wr_id;
                    qp->st.rnr_attempts = 0;
                    qp->st.rnr_next_ns = 0;
                } else {
                    // timeout, retry_cnt, rnr_retry, min_rnr_timer share one 32-bit word.
                    const uint8_t rnr_retry = uint8_t(ld_vol32(&qp->cfg.timeout) >> 16);
                    if (rnr_retry == 7) {
                        rnr = 1;
                    } else {
                        const uint64_t now = gtime();
                        if (qp->st.rnr_next_ns == 0 || now >= qp->st.rnr_next_ns) {
                            if (qp->st.rnr_next_ns != 0) qp->st.rnr_attempts += 1;
                            if (qp->st.rnr_attempts >= rnr_retry) {
                                rnr = 2;
                            } else {
                                const uint32_t code = ld_acq_sys32(&peer->cfg.timeout) >> 24;
                                qp->st.rnr_next_ns = now + rnr_ns(code);
                                rnr = 1;
                            }
                        } else {
                            rnr = 1;
                        }
                    }
                }
            }
            rnr = bcast(rnr);
            if (rnr == 1) break;
            if (rnr == 2) {
                status = UGDR_WC_RNR_RETRY_EXC_ERR;
                if (w.lane == 0) {
                    rec->status = status;
                    qp->st.rnr_attempts = 0;
                    qp->st.rnr_next_ns = 0;
                }
            }
        }
        if (w.lane == 0) {
            rec->signaled = signaled ? 1u : 0u;
            atomicCAS(&w.p->stats->first_start_ns, 0ull, (unsigned long long)gtime());
        }
        bool issued = true;
        if (status == UGDR_WC_SUCCESS) {
            if (is_atomic(op) || total <= kInlineBytes) {
                run_inline(w, rec, wqe_smem, op, total, remote);
                if (w.lane == 0) atomicAdd(&w.p->stats->inline_runs, 1ull);
            } else {
                // Chunk so one WR spreads over about half the warps, within [16 KiB, 256 KiB]:
                // large enough that claims are rare next to the copy, small enough that a lone
                // WR still reaches most SMs.
                const uint64_t cb = total / (nwarps / 2 + 1);
                uint32_t chunk = kChunkMin;
                while (chunk < cb && chunk < kChunkMax) chunk <<= 1;
                const uint32_t n = uint32_t((total + chunk - 1) / chunk);
                bool ok = false;
                if (w.lane == 0) {
                    rec->nchunks = n;
                    __threadfence();
                    ok = publish_job(jr, bitmap, rec, n, chunk, w.gwarp + uint32_t(issue));
                    if (!ok) rec->nchunks = 0;
                    else atomicAdd(&w.p->stats->jobs_published, 1ull);
                }
                issued = bcast(ok ? 1 : 0) != 0;
            }
        }
        if (!issued) break;  // no job slot: retry next pass
        if (w.lane == 0) {
            __threadfence();
            qp->st.sq_issue = issue + 1;
        }
        __syncwarp();
        ++work;
        if (status != UGDR_WC_SUCCESS) break;  // stop issuing behind an error
    }
    return work;
}

// Warp 0 of every CTA is its leader: it services its own QPs and, about every microsecond,
// mirrors the global control words (job bitmap, QP-slot bound, exit / stop / drain state) into
// shared memory.  Warps 1..15 service their QPs and copy chunks, reading only the mirror when
// idle.  Without the mirror every warp of the grid polled the same few L2 lines and every
// data access hashing to those slices queued behind the polls.
__global__ void __launch_bounds__(kThreads, 1) executor_kernel(ExecParams p) {
    __shared__ __align__(16) uint8_t wqe_buf[kWarps][kWqeBytesMax];
    __shared__ volatile uint32_t s_bits[32];
    __shared__ volatile uint32_t s_slots, s_exit, s_work;
    Warp w;
    w.p = &p;
    w.lane = threadIdx.x & 31;
    w.wi = threadIdx.x >> 5;
    w.gwarp = blockIdx.x * kWarps + w.wi;
    w.rot = w.gwarp * 2654435761u;
    w.abort = false;
    w.n_chunks = w.n_miss = w.bytes = w.busy = 0;
    const uint32_t nwarps = gridDim.x * kWarps;
    JobRing *jr = p.jobs;
    // Active-job bitmap: 32 words right after the ring (see job_ring_bytes()).
    uint32_t *bits = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(p.jobs) +
                                                  sizeof(JobRing));
    const uint64_t t_launch = gtime();
    const bool leader = w.wi == 0;
    if (threadIdx.x < 32) s_bits[threadIdx.x] = ld_vol32(&bits[threadIdx.x]);
    if (threadIdx.x == 0) {
        s_slots = ld_vol32(&p.stats->qp_slots);
        s_exit = 0;
        s_work = 0;
        if (blockIdx.x == 0) atomicAdd(&p.stats->launches_seen, 1ull);
    }
    __syncthreads();
    uint64_t t_refresh = t_launch, t_host = t_launch, t_pub = 0;
    uint32_t idle_rounds = 0;
    for (uint64_t iter = 0;; ++iter) {
        uint32_t work = 0;
        // Owned QPs: q = cta + grid * (wi + warps * k).
        const uint32_t slots = s_slots;
        const bool owner = blockIdx.x + gridDim.x * w.wi < slots;
        for (uint32_t q = blockIdx.x + gridDim.x * w.wi; q < slots; q += gridDim.x * kWarps) {
            work += service_qp(w, &p.qps[q], wqe_buf[w.wi], jr, bits, nwarps);
            if (w.abort) {
                s_exit = 1;
                flush_counters(w);
                return;
            }
        }
        if (!leader) {
            for (int k = 0; k < 8; ++k) {
                Claim cl;
                if (!claim_chunk(w, jr, bits, s_bits, &cl)) break;
                run_chunk(w, cl);
                ++work;
            }
            if (work != 0 && w.lane == 0) s_work = 1;
        } else {
            const uint64_t now = gtime();
            if (now - t_refresh >= 2000 || work != 0) {
                t_refresh = now;
                s_bits[w.lane] = ld_vol32(&bits[w.lane]);
                int exit_now = 0;
                if (w.lane == 0) {
                    s_slots = ld_vol32(&p.stats->qp_slots);
                    const bool busy = work != 0 || s_work != 0;
                    s_work = 0;
                    // Activity stamps are rare (one per CTA per 50 us) so the shared word
                    // stays cold.
                    if (busy && now - t_pub >= 50000) {
                        t_pub = now;
                        atomicMax(&p.stats->last_work_ns, (unsigned long long)now);
                    }
                    if (ld_vol32(&p.stats->exiting)) exit_now = 1;
                    if (blockIdx.x == 0) {
                        // The grid's control leader alone evaluates the exit conditions: the
                        // host stop flag (a PCIe read), drain completion and idleness.
                        if (now - t_host >= 10000) {
                            t_host = now;
                            if (ld_acq_sys32(const_cast<uint32_t *>(&p.ctrl->stop)) != 0) exit_now = 1;
                            if (p.mode == kPersistent && !busy) {
                                uint64_t last = ld_vol(&p.stats->last_work_ns);
                                if (last < t_launch) last = t_launch;
                                // Another CTA may have stamped a time later than `now`.
                                if (now > last && now - last > p.idle_exit_ns) exit_now = 1;
                            }
                        }
                        if (p.mode == kDrain && ld_vol(&p.stats->retired) >= p.expected) exit_now = 1;
                    }
                    if (exit_now) {
                        atomicExch(&p.stats->exiting, 1u);
                        s_exit = 1;
                    }
                }
                __syncwarp();
            }
        }
        if (s_exit) {
            flush_counters(w);
            return;
        }
        if ((iter & 1023) == 0) flush_counters(w);
        if (work == 0) {
            // QP owners poll quickly (latency); pure workers back off a little further.
            const uint32_t cap = owner ? 3u : 4u;
            idle_rounds = idle_rounds < 2 * cap ? idle_rounds + 1 : 2 * cap;
            __nanosleep(32u << (idle_rounds >> 1));
        } else {
            idle_rounds = 0;
        }
    }
}

// Copy-core unit kernel: one warp copies [src, src + n) to dst (alignment-matrix tests).
__global__ void copy_test_kernel(uint8_t *dst, const uint8_t *src, uint64_t n) {
    warp_copy(dst, src, n, threadIdx.x & 31);
}

// Copy-core ceiling: every warp of the grid copies one contiguous stripe with warp_copy, the
// same routine the executor's chunk workers run (no queues, no claims).
__global__ void __launch_bounds__(kThreads, 1) grid_copy_kernel(uint8_t *dst, const uint8_t *src,
                                                                 uint64_t n, uint64_t stripe) {
    const uint64_t gw = uint64_t(blockIdx.x) * kWarps + (threadIdx.x >> 5);
    const uint64_t off = gw * stripe;
    if (off >= n) return;
    const uint64_t len = n - off < stripe ? n - off : stripe;
    warp_copy(dst + off, src + off, len, threadIdx.x & 31);
}

}  // namespace

int launch_grid_copy(void *dst, const void *src, uint64_t n, int ctas, cudaStream_t stream) {
    const uint64_t warps = uint64_t(ctas) * kWarps;
    uint64_t stripe = (n + warps - 1) / warps;
    stripe = (stripe + 15) & ~uint64_t(15);
    grid_copy_kernel<<<ctas, kThreads, 0, stream>>>(static_cast<uint8_t *>(dst),
                                                    static_cast<const uint8_t *>(src), n, stripe);
    return int(cudaGetLastError());
}

size_t job_ring_bytes() { return sizeof(JobRing) + 32 * sizeof(uint32_t); }
int executor_threads() { return kThreads; }

int launch_executor(const ExecParams &p, int ctas, cudaStream_t stream) {
    executor_kernel<<<ctas, kThreads, 0, stream>>>(p);
    return int(cudaGetLastError());
}

int launch_copy_test(void *dst, const void *src, uint64_t n, cudaStream_t stream) {
    copy_test_kernel<<<1, 32, 0, stream>>>(static_cast<uint8_t *>(dst),
                                           static_cast<const uint8_t *>(src), n);
    return int(cudaGetLastError());
}

}  // namespace ugdr::gpu
