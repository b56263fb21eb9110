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
//  * Ownership.  QP slot q belongs to exactly one warp of the grid (CTA q % grid, owner rank
//    (q / grid) % warps, the CTA's leader warp ranked last; see owner_rank), so each QP's WRs are
//    fetched, validated and retired in posting order by one warp, and QPs spread over all SMs.
//  * Issue.  The owner warp reads up to 32 WQEs (host-mapped ring) lane-parallel into shared
//    memory, with up to 64 WRs of a QP in flight (two batches).  Single-SGE WRITE / READ are
//    validated lane-parallel (lane j checks WQE j against the device MR table); payloads up to
//    64 B are copied by their lane, larger ones become one chunked job for the whole batch.
//    Other WRs (multi-SGE, WRITE_WITH_IMM, atomics) are staged one after another and run inline
//    (<= 4 KiB, atomics) or join the pass's job.  Any warp of the GPU claims job chunks with a
//    fetch-and-add on the job's counter, so one large WR spreads over every SM.
//  * Retire.  When all chunks of the oldest in-flight WRs are done the owner produces the
//    receive CQEs (WRITE_WITH_IMM), the send CQEs (signaled or error) and advances the ring
//    head.  CQs are multi-producer (several warps, several GPUs): slots are reserved by CAS and
//    the tail moves in slot order, by turns passed through a device-memory tail hint (see
//    publish_cq), never by polling the host ring.
//  * Bounded waits.  Every spin carries a %globaltimer deadline; on expiry the kernel records
//    the reason in DevStats::error_code and every warp exits.  There is no __trap, assert or
//    unbounded loop.  The kernel also exits after `idle_exit_ns` without work, on a host stop
//    flag, or (drain mode) once `expected` WRs retired; in-flight state lives in device memory
//    so a relaunch resumes where the previous launch stopped.
#include "gpu/device_abi.hpp"
#include "gpu/executor.hpp"
#include "ugdr/api.hpp"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ugdr::gpu {
namespace {

#ifndef UGDR_EXEC_WARPS
#define UGDR_EXEC_WARPS 8  // warps per executor CTA (one CTA per SM); 8 keeps every thread under 255 registers with no spills
#endif
constexpr int kWarps = UGDR_EXEC_WARPS;
constexpr int kThreads = kWarps * 32;
#ifndef UGDR_WQE_STAGE
#define UGDR_WQE_STAGE 2048
#endif
constexpr uint32_t kWqeStage = UGDR_WQE_STAGE;  // per-warp WQE staging: kWqeStage / 64 WQEs, or one wide one
#ifndef UGDR_LEADER_OWNS_LAST
#define UGDR_LEADER_OWNS_LAST 1
#endif
// Owner rank of warp `wi` among its CTA's warps: QP q belongs to CTA q % grid and to the warp of
// rank (q / grid) % kWarps.  With UGDR_LEADER_OWNS_LAST the leader (warp 0, which also mirrors
// the control words) takes the last rank, so it owns a QP only when every other warp has one.
// Number of consecutive set bits from bit 0: 0..32 (`__ffs(~m) - 1` alone wraps when m is all ones).
__device__ __forceinline__ uint32_t ones_prefix(uint32_t m) { return m == 0xffffffffu ? 32u : uint32_t(__ffs(~m) - 1); }

__device__ __forceinline__ uint32_t owner_rank(uint32_t wi) {
    return UGDR_LEADER_OWNS_LAST ? (wi + kWarps - 1) % kWarps : wi;
}
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
__device__ __forceinline__ uint64_t ld_acq_gpu(const void *p) {
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t add_acq_gpu(void *p, uint64_t v) {
    uint64_t old;
    asm volatile("atom.acquire.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
    return old;
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
__device__ __forceinline__ void st_vol64(void *p, uint64_t v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
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
// Copies n bytes, never touching bytes outside [dst, dst + n) / [src, src + n).  32-byte vector
// body (sm_100 256-bit loads / stores, 4 in flight per lane) when both pointers share their
// offset mod 32 and the range is long; 16-byte body (8 in flight) when they share it mod 16;
// otherwise, from 64 bytes on, 16-byte stores built from shifted aligned 16-byte loads; bytes
// for short ranges.

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

// Bytes [r, r + 16) of the 32-byte concatenation a:b (0 < r < 16), as one 16-byte vector.
__device__ __forceinline__ uint4 shift_join(const uint4 &a, const uint4 &b, uint32_t r) {
    const uint32_t c[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const uint32_t sh = (r & 3) * 8;
    uint4 o;
    switch (r >> 2) {  // uniform across the warp: one branch, static register indices
    case 0:
        o = make_uint4(__funnelshift_r(c[0], c[1], sh), __funnelshift_r(c[1], c[2], sh), __funnelshift_r(c[2], c[3], sh),
                       __funnelshift_r(c[3], c[4], sh));
        break;
    case 1:
        o = make_uint4(__funnelshift_r(c[1], c[2], sh), __funnelshift_r(c[2], c[3], sh), __funnelshift_r(c[3], c[4], sh),
                       __funnelshift_r(c[4], c[5], sh));
        break;
    case 2:
        o = make_uint4(__funnelshift_r(c[2], c[3], sh), __funnelshift_r(c[3], c[4], sh), __funnelshift_r(c[4], c[5], sh),
                       __funnelshift_r(c[5], c[6], sh));
        break;
    default:
        o = make_uint4(__funnelshift_r(c[3], c[4], sh), __funnelshift_r(c[4], c[5], sh), __funnelshift_r(c[5], c[6], sh),
                       __funnelshift_r(c[6], c[7], sh));
        break;
    }
    return o;
}

__device__ void warp_copy(uint8_t *dst, const uint8_t *src, uint64_t n, int lane) {
    if (n == 0) return;
    const uintptr_t d = reinterpret_cast<uintptr_t>(dst), s = reinterpret_cast<uintptr_t>(src);
    if (((d ^ s) & 31) == 0 && n >= 4096) {
        const uint64_t head = (32 - (d & 31)) & 31;  // < 32 <= n
        if (uint64_t(lane) < head) dst[lane] = src[lane];
        dst += head;
        src += head;
        n -= head;
        const uint64_t nvec = n >> 5;
        V256 *dv = reinterpret_cast<V256 *>(dst);
        const V256 *sv = reinterpret_cast<const V256 *>(src);
        constexpr int U = 4;
        uint64_t i = lane;
        for (; i + (U - 1) * 32 < nvec; i += U * 32) {
            V256 r[U];
#pragma unroll
            for (int u = 0; u < U; ++u) r[u] = ld256(sv + i + u * 32);
#pragma unroll
            for (int u = 0; u < U; ++u) st256(dv + i + u * 32, r[u]);
        }
        for (; i < nvec; i += 32) st256(dv + i, ld256(sv + i));
        const uint64_t done = nvec << 5;
        if (uint64_t(lane) < n - done) dst[done + lane] = src[done + lane];
        return;
    }
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
    if (n >= 64) {
        // Source and destination disagree mod 16: align the destination, then build every
        // 16-byte destination vector from the two aligned source vectors that cover it (the
        // lane's own and its neighbour's, by shuffle), shifted by the constant misalignment r.
        // Loads stay 16-byte vectors with U steps in flight; an aligned source vector always
        // holds at least one byte of the range, so no load leaves the range's pages.
        const uint64_t head = (16 - (d & 15)) & 15;
        if (uint64_t(lane) < head) dst[lane] = src[lane];
        dst += head;
        src += head;
        n -= head;
        const uint32_t r = uint32_t(reinterpret_cast<uintptr_t>(src) & 15);  // != 0
        const uint4 *sa = reinterpret_cast<const uint4 *>(src - r);
        uint4 *dv = reinterpret_cast<uint4 *>(dst);
        const uint64_t nvec = n >> 4;
        constexpr int U = 4;  // 2 KiB in flight per warp: misaligned gathers are latency-bound
        for (uint64_t j0 = 0; j0 < nvec; j0 += 32 * U) {
            uint4 v[U], nx[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint64_t j = j0 + uint64_t(u) * 32 + lane;
                const uint64_t base = j0 + uint64_t(u) * 32;
                const uint64_t last = base + 31 < nvec ? base + 31 : nvec - 1;  // last vector of this step
                if (j < nvec) v[u] = ld128(sa + j);
                if (j == last) nx[u] = ld128(sa + j + 1);  // the step's last lane fetches its own next
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint64_t j = j0 + uint64_t(u) * 32 + lane;
                const uint64_t base = j0 + uint64_t(u) * 32;
                const uint64_t last = base + 31 < nvec ? base + 31 : nvec - 1;
                uint4 t;
                t.x = __shfl_down_sync(0xffffffffu, v[u].x, 1);
                t.y = __shfl_down_sync(0xffffffffu, v[u].y, 1);
                t.z = __shfl_down_sync(0xffffffffu, v[u].z, 1);
                t.w = __shfl_down_sync(0xffffffffu, v[u].w, 1);
                if (j == last) t = nx[u];
                if (j < nvec) st128(dv + j, shift_join(v[u], t, r));
            }
        }
        const uint64_t done = nvec << 4;
        if (uint64_t(lane) < n - done) dst[done + lane] = src[done + lane];
        return;
    }
    for (uint64_t i = lane; i < n; i += 32) dst[i] = src[i];
}

// ---- TMA bulk-copy path ----------------------------------------------------------------------
// Long 16-byte aligned pieces of a chunk move through the TMA bulk-copy engine instead of the
// load/store core: lane 0 of a chunk worker issues cp.async.bulk global -> shared (completion on
// an mbarrier, expected bytes) and shared -> global (bulk groups) over kTmaStages 4 KiB stages of
// its warp's own shared memory.  Untiled copies, no tensor map and no multicast: the source may be
// local or a peer's memory (READ), the destination local or a peer's (WRITE).  A bulk copy keeps
// far more bytes in flight per warp than the vector core, which is what an NVLink round trip
// wants.  Every mbarrier wait is bounded; when one runs out the copy waits (bounded) for its other
// loads, reports failure and the kernel exits with kErrBulkCopyTimeout.
#ifndef UGDR_TMA_STAGES
#define UGDR_TMA_STAGES 4  // 0 builds the executor without the bulk-copy path (no dynamic smem)
#endif
constexpr uint32_t kTmaStages = UGDR_TMA_STAGES > 0 ? UGDR_TMA_STAGES : 1;
constexpr bool kTmaBuilt = UGDR_TMA_STAGES > 0;
constexpr uint32_t kTmaPiece = 4096;

struct Tma {
    uint8_t *buf;    // kTmaStages x kTmaPiece bytes of this warp's shared memory
    uint64_t *bar;   // kTmaStages mbarriers, arrival count 1
    uint32_t phase;  // bit s: parity of stage s's next completion (lane 0)
    uint32_t min;    // pieces shorter than this stay on the load/store path
    uint32_t failed;
    uint64_t max_ns;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ bool mbar_wait_until(uint64_t *bar, uint32_t parity, uint64_t deadline) {
    for (uint32_t spins = 0;; ++spins) {
        uint32_t done = 0;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        if (done) return true;
        if ((spins & 15) == 15 && gtime() > deadline) return false;
    }
}
__device__ __forceinline__ void tma_load(Tma *t, uint32_t s, const uint8_t *src, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&t->bar[s])), "r"(bytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(t->buf + size_t(s) * kTmaPiece)),
        "l"(src), "r"(bytes), "r"(smem_u32(&t->bar[s]))
        : "memory");
}
__device__ __forceinline__ void tma_store(uint8_t *dst, const uint8_t *smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(smem)),
                 "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Lane 0: copy n bytes (dst, src and n multiples of 16) through the stages.  Returns false when a
// wait ran out (the stages are then left quiet, or as quiet as a second bounded wait allows).
__device__ bool tma_copy(Tma *t, uint8_t *dst, const uint8_t *src, uint64_t n) {
    // Generic-proxy writes to the source (earlier WRs) before the async proxy reads it.
    asm volatile("fence.proxy.async.global;" ::: "memory");
    const uint64_t pieces = (n + kTmaPiece - 1) / kTmaPiece;
    auto piece_bytes = [&](uint64_t i) {
        const uint64_t left = n - i * kTmaPiece;
        return uint32_t(left < kTmaPiece ? left : kTmaPiece);
    };
    uint64_t loaded = 0;
    for (; loaded < pieces && loaded < kTmaStages; ++loaded)
        tma_load(t, uint32_t(loaded % kTmaStages), src + loaded * kTmaPiece, piece_bytes(loaded));
    const uint64_t deadline = gtime() + t->max_ns;
    bool ok = true;
    uint64_t i = 0;
    for (; i < pieces; ++i) {
        const uint32_t s = uint32_t(i % kTmaStages);
        if (!mbar_wait_until(&t->bar[s], (t->phase >> s) & 1u, deadline)) {
            ok = false;
            break;
        }
        t->phase ^= 1u << s;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tma_store(dst + i * kTmaPiece, t->buf + size_t(s) * kTmaPiece, piece_bytes(i));
        if (loaded < pieces) {
            // Stage s is refilled only once the store just issued has read it.
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            tma_load(t, s, src + loaded * kTmaPiece, piece_bytes(loaded));
            ++loaded;
        }
    }
    if (!ok) {
        const uint64_t d2 = gtime() + t->max_ns;
        for (uint64_t j = i; j < loaded; ++j) {
            const uint32_t s = uint32_t(j % kTmaStages);
            if (mbar_wait_until(&t->bar[s], (t->phase >> s) & 1u, d2)) t->phase ^= 1u << s;
        }
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    // The bulk stores are complete; order them before the generic-proxy release that follows.
    asm volatile("fence.proxy.async.global;" ::: "memory");
    return ok;
}

// Warp-wide copy of one range: the aligned body through the TMA when it is long enough, the rest
// (or all of it) with the vector core.
__device__ void range_copy(Tma *t, uint8_t *dst, const uint8_t *src, uint64_t n, int lane) {
    if (t != nullptr && t->min != 0 && ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0 &&
        n >= t->min) {
        const uint64_t body = n & ~uint64_t(15);
        int ok = 1;
        if (lane == 0) ok = tma_copy(t, dst, src, body) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) t->failed = 1;
        warp_copy(dst + body, src + body, n - body, lane);
        return;
    }
    warp_copy(dst, src, n, lane);
}

// Copy stream bytes [off, off + len) of a WR: local segments <-> contiguous remote range.
// `t` (null: none) is the calling warp's TMA staging.
__device__ __noinline__ void copy_stream(const WrRec *rec, uint32_t nseg, uint64_t remote, bool to_remote,
                                         uint64_t off, uint64_t len, int lane, Tma *t) {
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
            range_copy(t, to_remote ? rem : local, to_remote ? local : rem, take, lane);
            off += take;
            len -= take;
        }
        seg_start += sl;
    }
}

// ---- elementwise bf16 sum (UGDR_X_WR_RDMA_WRITE_SUM_BF16) ----------------------------------------
// Bytes [off, off + len) of the destination get the fp32 sum, in SGE order, of the same bytes of
// every segment (all segments have the WR's length), rounded to bf16.  Each lane reads all inputs
// of its elements before it writes them, so the destination may be one of the segments.

__device__ __forceinline__ void acc_bf16x2(float &lo, float &hi, uint32_t x) {
    lo += __uint_as_float(x << 16);
    hi += __uint_as_float(x & 0xffff0000u);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// Multicast (NVLS) forms, for WRs whose source or destination MR is an NVLink multicast view:
// the load has the NVSwitch read the 16 bytes from every GPU bound to the object and return the
// fp32-accumulated bf16 sums; the store writes 16 bytes to every one of them.
__device__ __forceinline__ uint4 mc_ld_sum(const uint8_t *p) {
    uint4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}
__device__ __forceinline__ void mc_st(uint8_t *p, uint4 v) {
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// WrRec::pad[0] bits of a WRITE_SUM_BF16 whose MRs are multicast views (stage_wr checks that
// such a WR has one SGE and 16-byte aligned addresses and length).
constexpr uint32_t kWrSrcMulticast = 1, kWrDstMulticast = 2;

__device__ __noinline__ void sum_stream_mc(uint32_t mc, const WrRec *rec, uint64_t remote, uint64_t off, uint64_t len, int lane) {
    const uint8_t *src =
        reinterpret_cast<const uint8_t *>(__ldcg(reinterpret_cast<const unsigned long long *>(&rec->seg[0].local))) + off;
    uint8_t *dst = reinterpret_cast<uint8_t *>(remote) + off;
    // Unicast writes of the inputs (earlier WRs, other GPUs) before the multicast reads.
    asm volatile("fence.proxy.alias;" ::: "memory");
    const uint64_t nvec = len >> 4;
    constexpr int U = 4;
    for (uint64_t v0 = lane; v0 < nvec; v0 += 32 * U) {
        uint4 x[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t v = v0 + uint64_t(u) * 32;
            if (v < nvec) x[u] = (mc & kWrSrcMulticast) ? mc_ld_sum(src + v * 16) : ld128(src + v * 16);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t v = v0 + uint64_t(u) * 32;
            if (v >= nvec) continue;
            if (mc & kWrDstMulticast)
                mc_st(dst + v * 16, x[u]);
            else
                st128(dst + v * 16, x[u]);
        }
    }
    // The multicast stores before the retire's fences and the peers' unicast reads of the result.
    asm volatile("fence.proxy.alias;" ::: "memory");
}

__device__ __noinline__ void sum_stream(const WrRec *rec, uint32_t nseg, uint64_t remote, uint64_t off,
                                        uint64_t len, int lane) {
    if (const uint32_t mc = __ldcg(&rec->pad[0]); mc != 0) {
        sum_stream_mc(mc, rec, remote, off, len, lane);
        return;
    }
    // Lane i holds segment i's source address at `off`; the others come by shuffle.
    const uint64_t mine =
        uint32_t(lane) < nseg
            ? uint64_t(__ldcg(reinterpret_cast<const unsigned long long *>(&rec->seg[lane].local))) + off
            : 0;
    uint8_t *dst = reinterpret_cast<uint8_t *>(remote) + off;
    const uint32_t misaligned =
        __ballot_sync(0xffffffffu, (uint32_t(lane) < nseg && (mine & 15) != 0) || (lane == 0 && (uintptr_t(dst) & 15)));
    const uint64_t nvec = misaligned ? 0 : len >> 4;
    // Loop bounds are uniform over the warp, so every lane reaches each shuffle: full groups of
    // 64 vectors (two per lane in flight), then groups of 32 with the lanes past the end idle.
    uint64_t base = 0;
    for (; base + 64 <= nvec; base += 64) {
        const uint64_t v = base + lane;
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (uint32_t i = 0; i < nseg; ++i) {
            const uint8_t *src = reinterpret_cast<const uint8_t *>(__shfl_sync(0xffffffffu, (unsigned long long)mine, i));
            const uint4 x = ld128(src + v * 16), y = ld128(src + (v + 32) * 16);
            acc_bf16x2(a[0], a[1], x.x);
            acc_bf16x2(a[2], a[3], x.y);
            acc_bf16x2(a[4], a[5], x.z);
            acc_bf16x2(a[6], a[7], x.w);
            acc_bf16x2(b[0], b[1], y.x);
            acc_bf16x2(b[2], b[3], y.y);
            acc_bf16x2(b[4], b[5], y.z);
            acc_bf16x2(b[6], b[7], y.w);
        }
        st128(dst + v * 16, make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]), pack_bf16x2(a[4], a[5]),
                                       pack_bf16x2(a[6], a[7])));
        st128(dst + (v + 32) * 16, make_uint4(pack_bf16x2(b[0], b[1]), pack_bf16x2(b[2], b[3]),
                                              pack_bf16x2(b[4], b[5]), pack_bf16x2(b[6], b[7])));
    }
    for (; base < nvec; base += 32) {
        const uint64_t v = base + lane;
        const bool in = v < nvec;
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (uint32_t i = 0; i < nseg; ++i) {
            const uint8_t *src = reinterpret_cast<const uint8_t *>(__shfl_sync(0xffffffffu, (unsigned long long)mine, i));
            if (!in) continue;
            const uint4 x = ld128(src + v * 16);
            acc_bf16x2(a[0], a[1], x.x);
            acc_bf16x2(a[2], a[3], x.y);
            acc_bf16x2(a[4], a[5], x.z);
            acc_bf16x2(a[6], a[7], x.w);
        }
        if (in)
            st128(dst + v * 16, make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]), pack_bf16x2(a[4], a[5]),
                                           pack_bf16x2(a[6], a[7])));
    }
    // Tail, or everything when an address is not 16-byte aligned: 2-byte elements.  The loop
    // bound is uniform over the warp so every lane reaches each shuffle.
    const uint64_t e0 = (nvec << 4) >> 1, ne = len >> 1;
    for (uint64_t base = e0; base < ne; base += 32) {
        const uint64_t e = base + lane;
        float acc = 0.f;
        for (uint32_t i = 0; i < nseg; ++i) {
            const uint8_t *src = reinterpret_cast<const uint8_t *>(__shfl_sync(0xffffffffu, (unsigned long long)mine, i));
            if (e < ne) acc += __uint_as_float(uint32_t(*reinterpret_cast<const uint16_t *>(src + 2 * e)) << 16);
        }
        if (e < ne) {
            const __nv_bfloat16 r = __float2bfloat16_rn(acc);
            *reinterpret_cast<__nv_bfloat16 *>(dst + 2 * e) = r;
        }
    }
}

// ---- per-launch warp context -------------------------------------------------------------------

// A QP's configuration as one service pass sees it (read once per pass, in parallel).
struct QpView {
    queue::RingHeader *sq;
    const uint8_t *sq_slots;
    DevQp *peer;
    DevCq *send_cq;
    uint32_t sq_cap, sq_stride, qpn, state, pd, max_sge, sig_all, lost, err, err_issued, retry_word;
    // Responder configuration as of the last refresh (at most 20 us old).
    uint32_t pstate, perr, pactive, pacc, ppd;
};

// Per-warp cache of the two MR entries the fast path used last.  An entry hits only under the
// MR epoch it was cached in: deregistration bumps the epoch after it invalidates the table entry,
// and a key's generation bits make a reused slot miss.
struct MrCacheEntry {
    uint32_t key, epoch, pad[2];  // epoch: DevStats::mr_epoch when cached (a newer one misses)
    uint4 part[3];
};

// A warp's cached view of the last CQ it produced into (configuration never changes while the
// CQ is attached; the cursors are guesses that a failed CAS corrects).
struct CqCache {
    DevCq *cq;
    queue::RingHeader *ring;
    uint8_t *slots;
    uint32_t cap, stride;
    unsigned long long *ready;
    uint64_t reserve, head, published;
    uint32_t epoch;  // MR epoch when filled: a CQ slot is reused only under a newer one
};

// A warp's private statistics, folded into DevStats now and then (hot shared counters would
// serialise every warp of the grid on one L2 line).  Kept in shared memory, not registers.
struct WarpCounters {
    unsigned long long n_chunks, n_miss, bytes, busy, n_inline, n_slow, t_slow, n_slot_miss, n_pub_wait, t_pub_wait;
};

struct Warp {
    const ExecParams *p;
    int lane;
    uint32_t wi;    // warp index inside the CTA
    uint32_t gwarp; // global warp index
    uint32_t rot;   // job-slot rotation seed
    bool abort;
    // Private counters, folded into DevStats now and then (hot shared counters would serialise
    // every warp of the grid on one L2 line).
    WarpCounters *ctr;  // this warp's counters (shared memory, updated by lane 0)
    bool started;  // this warp stamped first_start_ns in this launch
    CqCache *cq;  // lane 0's cache of the last CQ it produced into (shared memory)
    MrCacheEntry *mrc;  // this warp's two-entry MR cache (shared memory)
    volatile uint32_t *mirror;  // the CTA's shared copy of the active-job bitmap
    // Cached view of the QP this warp serviced last (see service_qp).
    DevQp *vq;
    uint64_t vt, vhead, vissue, vtail, t_reserved;
    uint32_t vepoch;  // MR epoch the view was read under: a newer epoch forces a re-read
    QpView *vv;  // cached view of the QP serviced last (shared memory)
    Tma *tma;    // this warp's TMA staging (null for the leader warp, which runs no chunks)
    volatile uint32_t *mr_epoch;  // the CTA's shared copy of DevStats::mr_epoch
    uint32_t epoch;               // the MR epoch of the current service pass
};

// Appends one trace record (lane 0 only; the caller checks that tracing is on).  Not inlined:
// the hot paths keep only the null test of p->trace.
__device__ __noinline__ void trace_event(const ExecParams *p, uint32_t ev, uint32_t gwarp, uint32_t qp,
                                         uint32_t value, uint64_t t0, uint64_t t1) {
    const uint32_t i = atomicAdd(&p->trace_count[blockIdx.x], 1u);
    if (i >= p->trace_cap) return;
    TraceRec *r = p->trace + size_t(blockIdx.x) * p->trace_cap + i;
    r->t0 = t0;
    r->t1 = t1;
    r->event = (ev << 16) | (gwarp & 0xffffu);
    r->qp = qp;
    r->value = value;
    r->cta = blockIdx.x;
}

__device__ void record_error(Warp &w, uint32_t code) {
    if (w.lane == 0) {
        if (w.p->trace != nullptr) trace_event(w.p, kTraceError, w.gwarp, 0xffffffffu, code, gtime(), gtime());
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

// Reserve up to `want` consecutive slots of a multi-producer CQ (lane 0).  Returns how many were
// granted (0 when the CQ is full); *first receives the first slot's cursor.  The warp caches the
// CQ's configuration and its last view of the cursors, so an uncontended reservation is one CAS.
__device__ uint32_t reserve_cq(Warp &w, DevCq *cq, uint32_t want, uint64_t *first) {
    CqCache &c = *w.cq;
    if (c.cq != cq || c.epoch != w.epoch) {
        c.cq = cq;
        c.epoch = w.epoch;
        c.cap = ld_vol32(&cq->cfg.capacity);
        c.stride = ld_vol32(&cq->cfg.stride);
        c.ring = reinterpret_cast<queue::RingHeader *>(ld_vol(&cq->cfg.ring));
        c.slots = reinterpret_cast<uint8_t *>(ld_vol(&cq->cfg.slots));
        c.ready = reinterpret_cast<unsigned long long *>(ld_vol(&cq->cfg.ready));
        c.reserve = ld_vol(&cq->st.reserve);
        c.head = ld_vol(&cq->st.head_seen);
        c.published = ~0ull;
    }
    for (int attempt = 0; attempt < 256; ++attempt) {
        const uint64_t r = c.reserve;
        if (r - c.head + want > c.cap) {
            const uint64_t head = ld_acq_sys(&c.ring->head.value);  // the consumer moved on
            if (head > c.head) c.head = head;
            atomicMax_system(&cq->st.head_seen, c.head);
        }
        const uint64_t used = r - c.head;
        if (used >= c.cap) {
            c.cq = nullptr;  // re-read everything next time
            return 0;
        }
        const uint32_t k = uint32_t(want < c.cap - used ? want : c.cap - used);
        const uint64_t old = atomicCAS_system(&cq->st.reserve, r, r + k);
        if (old == r) {
            c.reserve = r + k;
            *first = r;
            return k;
        }
        c.reserve = old;  // another producer got there first: retry from its cursor
    }
    c.cq = nullptr;
    return 0;
}

// ---- CQ publication ---------------------------------------------------------------------------
// A CQ may have many producers (warps on this and other GPUs).  Slots are reserved in order
// (reserve_cq) but written by whoever reserved them; the ring tail must advance in slot order and
// only over written slots.  DevCqState::published is a device-memory hint of the tail, and the
// producer that owns slot `published` is the only one that may move the tail ("its turn"):
//  * a producer writes its CQEs, fences them (system scope) and tags each of its slots s with
//    s + 1 in the device-memory `ready` array;
//  * it polls `published` (GPU memory, not the host ring over PCIe) until it reaches its slots;
//    if a predecessor already moved the tail past them it is done;
//  * on its turn it first reads the host tail until the predecessor's tail store has landed
//    (usually at once), so tail stores are coherence-ordered and the tail never moves back; then
//    it extends its range over every consecutively tagged slot after its own - waiting
//    successors - and stores the host tail and the hint once for the whole batch.
// A producer that stored the tail last and reserved the next slots (one producer streaming into
// its CQ) skips the tags and both polls: fence, tail store, hint store.
__device__ bool publish_cq(Warp &w, DevCq *cq, uint64_t first, const queue::Cqe *e, uint32_t k, uint64_t max_ns) {
    CqCache &c = *w.cq;
    for (uint32_t i = 0; i < k; ++i) {
        uint8_t *slot = c.slots + ((first + i) % c.cap) * c.stride;
        const uint4 *src = reinterpret_cast<const uint4 *>(&e[i]);
        st_vol128(slot, src[0]);
        st_vol128(slot + 16, src[1]);
    }
    // One system fence orders the WR payload stores and the CQE slots before the tail (or the
    // tags another producer publishes them by).
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    uint64_t from = first;
    if (c.published != first) {
        for (uint32_t i = 0; i < k; ++i) st_vol64(&c.ready[(first + i) % c.cap], first + i + 1);
        const uint64_t t0 = gtime();
        uint32_t spins = 0;
        uint64_t p;
        while ((p = ld_acq_sys(&cq->st.published)) < first) {
            if ((++spins & 63) == 0 && gtime() - t0 > max_ns) return false;
            __nanosleep(32);
        }
        if (p >= first + k) {
            if (w.lane == 0) w.ctr->n_pub_wait += 1;
            if (w.lane == 0) w.ctr->t_pub_wait += gtime() - t0;
            c.published = p;  // a predecessor published these slots
            return true;
        }
        from = p;  // our turn (part of our range may already be out)
        if (!wait_eq_sys(reinterpret_cast<const unsigned long long *>(&c.ring->tail.value), from, max_ns))
            return false;
        if (w.lane == 0) w.ctr->n_pub_wait += 1;
        if (w.lane == 0) w.ctr->t_pub_wait += gtime() - t0;
    }
    uint64_t end = first + k;
    while (end - from < c.cap && ld_acq_sys(&c.ready[end % c.cap]) == end + 1) ++end;
    st_vol64(&c.ring->tail.value, end);
    st_vol64(&cq->st.published, end);
    c.published = end;
    return true;
}

// One CQE, reserved and published (lane 0): 0 published, 1 CQ full, 2 publish wait ran out.
__device__ int produce_cqe(Warp &w, DevCq *cq, const queue::Cqe &e, uint64_t max_ns) {
    uint64_t r = 0;
    if (reserve_cq(w, cq, 1, &r) == 0) return 1;
    return publish_cq(w, cq, r, &e, 1, max_ns) ? 0 : 2;
}

// Claim the next RQ WR of `qp` (lane 0).  Returns false when the RQ is empty.
__device__ bool claim_rq(DevQp *qp, uint64_t *claim, uint64_t *wr_id) {
    queue::RingHeader *rq = reinterpret_cast<queue::RingHeader *>(ld_vol(&qp->cfg.rq));
    for (int attempt = 0; attempt < 64; ++attempt) {
        const uint64_t c = ld_vol(&qp->st.rq_claim);
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
// ---- ordering within a QP --------------------------------------------------------------------
// The WRs of one QP take effect in posting order (RC semantics: the responder executes them in
// order, so of two WRITEs to the same bytes the later one wins, and a READ sees every earlier
// WRITE).  The executor runs a batch's WRs on different lanes at once, and large WRs as chunked
// jobs that finish later, so a WR starts only when no earlier WR of its QP that may still be
// moving bytes touches the same bytes with at least one of the two writing them.  Addresses are
// device addresses in this GPU's mappings; every registered allocation is mapped once per GPU,
// so the same bytes always have the same address here.

// The bytes one WR touches: the remote range [rl, rh) and the extent of its local segments
// [ll, lh); w bit 0: the remote range is written, bit 1: the local range is written.
struct Span {
    uint64_t rl, rh, ll, lh;
    uint32_t w;
};

__device__ __forceinline__ Span span_of(uint32_t op, uint64_t remote, uint64_t total, uint64_t lo, uint64_t hi,
                                        bool moves) {
    Span s{0, 0, 0, 0, 0};
    if (!moves) return s;
    s.rl = remote;
    s.rh = remote + (is_atomic(op) ? 8 : total);
    s.ll = lo;
    s.lh = hi;
    s.w = op == UGDR_WR_RDMA_READ ? 2u : is_atomic(op) ? 3u : 1u;
    return s;
}

__device__ __forceinline__ bool overlap(uint64_t al, uint64_t ah, uint64_t bl, uint64_t bh) {
    return al < bh && bl < ah;
}

// True when a and b touch a common byte and at least one of them writes it.
__device__ __forceinline__ bool clash(const Span &a, const Span &b) {
    const bool awr = a.w & 1u, awl = a.w & 2u, bwr = b.w & 1u, bwl = b.w & 2u;
    return (overlap(a.rl, a.rh, b.rl, b.rh) && (awr || bwr)) || (overlap(a.rl, a.rh, b.ll, b.lh) && (awr || bwl)) ||
           (overlap(a.ll, a.lh, b.rl, b.rh) && (awl || bwr)) || (overlap(a.ll, a.lh, b.ll, b.lh) && (awl || bwl));
}

__device__ __forceinline__ Span shfl_span(const Span &s, int src) {
    Span o;
    o.rl = __shfl_sync(0xffffffffu, (unsigned long long)s.rl, src);
    o.rh = __shfl_sync(0xffffffffu, (unsigned long long)s.rh, src);
    o.ll = __shfl_sync(0xffffffffu, (unsigned long long)s.ll, src);
    o.lh = __shfl_sync(0xffffffffu, (unsigned long long)s.lh, src);
    o.w = __shfl_sync(0xffffffffu, s.w, src);
    return o;
}

// Smallest and largest address any of the warp's spans touches (empty spans excluded).
__device__ __forceinline__ void span_box(const Span &s, uint64_t *lo, uint64_t *hi) {
    uint64_t a = ~0ull, b = 0;
    if (s.rl < s.rh) {
        a = s.rl;
        b = s.rh;
    }
    if (s.ll < s.lh) {
        a = s.ll < a ? s.ll : a;
        b = s.lh > b ? s.lh : b;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t ta = __shfl_xor_sync(0xffffffffu, (unsigned long long)a, o);
        const uint64_t tb = __shfl_xor_sync(0xffffffffu, (unsigned long long)b, o);
        a = ta < a ? ta : a;
        b = tb > b ? tb : b;
    }
    *lo = a;
    *hi = b;
}

// Warp-wide: true on the lanes whose span clashes with a WR of `qp` in [head, issue) (issued,
// not yet retired; such a WR may still be copying).  Lane k loads WR head + k's record.
__device__ bool clashes_in_flight(const Warp &w, DevQp *qp, uint64_t head, uint64_t issue, const Span &mine) {
    const uint32_t all = uint32_t(issue - head);
    if (all == 0 || __all_sync(0xffffffffu, mine.w == 0)) return false;
    bool hit = false;
    for (uint32_t base = 0; base < all; base += 32) {  // in-flight WRs, 32 at a time (lane k: WR base + k)
        const uint32_t m = all - base < 32 ? all - base : 32u;
        Span f{0, 0, 0, 0, 0};
        if (uint32_t(w.lane) < m) {
            const WrRec *r = &qp->st.win[(head + base + w.lane) % kWindow];
            if (ld_vol32(&r->status) == UGDR_WC_SUCCESS)
                f = span_of(ld_vol32(&r->opcode), ld_vol(&r->remote), ld_vol(&r->total), ld_vol(&r->lo),
                            ld_vol(&r->hi), true);
        }
        // Cheap filter: nothing of these reaches the addresses this warp's spans touch.
        uint64_t blo, bhi;
        span_box(f, &blo, &bhi);
        const bool near =
            mine.w != 0 && (overlap(mine.rl, mine.rh, blo, bhi) || overlap(mine.ll, mine.lh, blo, bhi));
        if (!__any_sync(0xffffffffu, near)) continue;
        for (uint32_t k = 0; k < m; ++k) {
            const Span s = shfl_span(f, int(k));
            hit |= mine.w != 0 && clash(s, mine);
        }
    }
    return hit;
}

// Warp-wide: true on lane j (< n) when its span clashes with the span of a lane i < j.
__device__ bool clashes_in_batch(const Warp &w, uint32_t n, const Span &mine) {
    if (n < 2) return false;
    // Cheap filter: written ranges ascending and disjoint lane by lane, and the written and read
    // ranges of the batch in disjoint address boxes.  Both hold for the usual streaming pattern.
    const uint64_t wl = (mine.w & 1u) ? mine.rl : (mine.w & 2u) ? mine.ll : 0;
    const uint64_t wh = (mine.w & 1u) ? mine.rh : (mine.w & 2u) ? mine.lh : 0;
    const uint64_t rl = (mine.w & 1u) ? mine.ll : mine.rl, rh = (mine.w & 1u) ? mine.lh : mine.rh;
    const bool two_writes = mine.w == 3u;
    uint64_t pmax = wh;  // inclusive prefix max of written ends, then made exclusive
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t t = __shfl_up_sync(0xffffffffu, (unsigned long long)pmax, o);
        if (w.lane >= o && t > pmax) pmax = t;
    }
    uint64_t prev = __shfl_up_sync(0xffffffffu, (unsigned long long)pmax, 1);
    if (w.lane == 0) prev = 0;
    const bool in = uint32_t(w.lane) < n;
    bool suspect = in && (two_writes || (wl < wh && wl < prev));
    uint64_t wlo = in && wl < wh ? wl : ~0ull, whi = in && wl < wh ? wh : 0;
    uint64_t rlo = in && rl < rh ? rl : ~0ull, rhi = in && rl < rh ? rh : 0;
    for (int o = 16; o > 0; o >>= 1) {
        uint64_t t = __shfl_xor_sync(0xffffffffu, (unsigned long long)wlo, o);
        wlo = t < wlo ? t : wlo;
        t = __shfl_xor_sync(0xffffffffu, (unsigned long long)whi, o);
        whi = t > whi ? t : whi;
        t = __shfl_xor_sync(0xffffffffu, (unsigned long long)rlo, o);
        rlo = t < rlo ? t : rlo;
        t = __shfl_xor_sync(0xffffffffu, (unsigned long long)rhi, o);
        rhi = t > rhi ? t : rhi;
    }
    if (!__any_sync(0xffffffffu, suspect) && !overlap(wlo, whi, rlo, rhi)) return false;
    bool hit = false;
    for (uint32_t i = 0; i + 1 < n; ++i) {
        const Span s = shfl_span(mine, int(i));
        hit |= in && uint32_t(w.lane) > i && clash(s, mine);
    }
    return hit;
}

__device__ uint64_t rnr_ns(uint32_t code) {
    constexpr uint32_t t[32] = {65536, 1,    2,    3,    4,    6,    8,     12,    16,   24,   32,
                            48,    64,   96,   128,  192,  256,  384,   512,   768,  1024, 1536,
                            2048,  3072, 4096, 6144, 8192, 12288, 16384, 24576, 32768, 49152};
    return uint64_t(t[code & 31]) * 10000ull;
}

// ---- jobs ------------------------------------------------------------------------------------

// Take a free job slot (lane 0).  Returns its index (and the job generation it starts), or -1
// when none is free.
__device__ int take_job_slot(JobRing *jr, uint32_t seed, unsigned long long *gen) {
    for (uint32_t k = 0; k < 64; ++k) {
        const uint32_t s = (seed * 37u + k * 97u) % kJobSlots;
        Job *j = &jr->slots[s];
        // Slot free <=> seq even; taking it makes seq odd.  gen = (seq + 1) / 2 is new each time.
        const unsigned long long seq = ld_vol(&j->seq);
        if ((seq & 1ull) != 0) continue;
        if (atomicCAS(&j->seq, seq, seq + 1) != seq) continue;
        *gen = (seq + 1) >> 1;
        return int(s);
    }
    return -1;
}

// Publish WRs [first, first + nwr) of a QP window as one job in a taken slot (warp-wide): lane
// i (< nwr) passes WR i's first chunk index.  The WRs' records are complete before the call.
// The CTA's own bitmap mirror is updated at once so its warps can start claiming immediately;
// other CTAs see the job at their leader's next refresh.
__device__ void publish_job(Warp &w, JobRing *jr, uint32_t *bitmap, int slot, unsigned long long gen,
                            WrRec *win, uint32_t first, uint32_t nwr, uint32_t start, uint32_t nchunks,
                            uint32_t chunk_bytes) {
    Job *j = &jr->slots[slot];
    if (uint32_t(w.lane) < nwr) j->start[w.lane] = start;
    if (w.lane == 0) {
        j->win = win;
        j->nchunks = nchunks;
        j->chunk_bytes = chunk_bytes;
        j->first = first;
        j->nwr = nwr;
        j->done = 0;
    }
    __syncwarp();
    if (w.lane == 0) {
        __threadfence();
        atomicExch(&j->ctl, gen << 32);
        __threadfence();
        const uint32_t bit = 1u << (slot & 31);
        atomicOr(&bitmap[slot >> 5], bit);
        atomicOr(const_cast<uint32_t *>(&w.mirror[slot >> 5]), bit);
        atomicAdd(&w.p->stats->jobs_published, 1ull);
    }
    __syncwarp();
}

struct Claim {
    WrRec *rec;
    Job *job;
    uint64_t off;
    uint32_t cb, n;
};

// Claim one chunk from any active job (warp-wide): a fetch-and-add on the job's counter, which
// always yields a unique index (no CAS retry storms when thousands of warps contend).
//  * The fields are read after an acquiring load of the counter; if the add returns the same
//    generation, no recycle happened in between, so the fields belong to it (a slot is recycled
//    only after all of its chunks are done, which cannot be while our index is below nchunks).
//  * If the add lands in a newer generation, the index belongs to that job: re-read its fields
//    (stable for the same reason) and run it, so no index is ever lost.
// The chunk's WR is found by a ballot over the job's per-WR start indices, one per lane.
// `mirror` is the CTA's shared copy of the active-job bitmap (refreshed by the CTA leader).
__device__ bool claim_chunk(Warp &w, JobRing *jr, uint32_t *bitmap, const volatile uint32_t *mirror,
                            Claim *out) {
    const uint32_t word = mirror[w.lane];
    const uint32_t nonzero = __ballot_sync(0xffffffffu, word != 0);
    if (nonzero == 0) return false;
    int got = 0;
    uint32_t c = 0, slot = 0;
    uint4 g{};
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
            slot = wsel * 32 + b;
            Job *j = &jr->slots[slot];
            const unsigned long long v0 = ld_acq_gpu(&j->ctl);
            const uint4 f = ld_vol128(&j->win);  // win (x,y), nchunks (z), chunk_bytes (w)
            if (uint32_t(v0) < f.z) {
                const unsigned long long v = add_acq_gpu(&j->ctl, 1ull);
                g = f;
                if ((v >> 32) != (v0 >> 32)) g = ld_vol128(&j->win);  // newer generation
                c = uint32_t(v);
                if (c < g.z) {
                    got = 1;
                    if (c + 1 == g.z) atomicAnd(&bitmap[wsel], ~(1u << b));  // all handed out
                }
            }
            // Every chunk of this job is handed out: drop it from the CTA's mirror so the other
            // warps here stop trying it before the leader's next refresh.
            if (!got) atomicAnd(const_cast<uint32_t *>(&w.mirror[wsel]), ~(1u << b));
        }
        w.rot = w.rot * 1664525u + 1013904223u;
    }
    w.rot = __shfl_sync(0xffffffffu, w.rot, 0);
    got = __shfl_sync(0xffffffffu, got, 0);
    if (!got) {
        if (w.lane == 0) w.ctr->n_miss += 1;
        return false;
    }
    __syncwarp();  // lane 0's acquire orders the other lanes' reads of the job below
    c = bcast(c);
    slot = bcast(slot);
    g.x = bcast(g.x);
    g.y = bcast(g.y);
    g.z = bcast(g.z);
    g.w = bcast(g.w);
    Job *j = &jr->slots[slot];
    const uint32_t first = ld_vol32(&j->first), nwr = ld_vol32(&j->nwr);
    const uint32_t st = uint32_t(w.lane) < nwr ? ld_vol32(&j->start[w.lane]) : 0xffffffffu;
    const uint32_t le = __ballot_sync(0xffffffffu, uint32_t(w.lane) < nwr && st <= c);
    const int wr = le ? 31 - __clz(le) : 0;
    const uint32_t s0 = __shfl_sync(0xffffffffu, st, wr);
    WrRec *win = reinterpret_cast<WrRec *>((uint64_t(g.y) << 32) | g.x);
    out->rec = win + (first + uint32_t(wr)) % kWindow;
    out->job = j;
    out->off = uint64_t(c - s0) * g.w;
    out->cb = g.w;
    out->n = g.z;
    return true;
}

__device__ void run_chunk(Warp &w, const Claim &cl) {
    WrRec *rec = cl.rec;
    const uint64_t total = ld_vol(&rec->total);
    const uint64_t off = cl.off;
    uint64_t len = total - off;
    if (len > cl.cb) len = cl.cb;
    const uint32_t op = ld_vol32(&rec->opcode);
    const uint32_t nseg = ld_vol32(&rec->nseg);
    const uint64_t remote = ld_vol(&rec->remote);
    const uint64_t t0 = gtime();
    if (op == UGDR_X_WR_RDMA_WRITE_SUM_BF16)
        sum_stream(rec, nseg, remote, off, len, w.lane);
    else
        copy_stream(rec, nseg, remote, op != UGDR_WR_RDMA_READ, off, len, w.lane, w.tma);
    __syncwarp();
    if (w.tma != nullptr && w.tma->failed) {
        record_error(w, kErrBulkCopyTimeout);
        return;  // the chunk stays unfinished: the kernel exits and reports the error
    }
    if (w.lane == 0) {
        // Device-scope release is enough here: the owner warp acquires chunks_done and issues
        // the system-scope fence before it publishes the CQE, and causality is transitive.
        __threadfence();
        atomicAdd(&rec->chunks_done, 1u);
        if (atomicAdd(&cl.job->done, 1u) + 1 == cl.n) atomicAdd(&cl.job->seq, 1ull);  // free the slot
    }
    if (w.lane == 0) {
        const uint64_t t1 = gtime();
        w.ctr->n_chunks += 1;
        w.ctr->bytes += len;
        w.ctr->busy += t1 - t0;
        if (w.p->trace != nullptr) trace_event(w.p, kTraceChunk, w.gwarp, 0xffffffffu, uint32_t(len), t0, t1);
    }
}

// Fold the warp's private counters into DevStats (lane 0).
__device__ void flush_counters(Warp &w) {
    if (w.lane == 0) {
        WarpCounters &c = *w.ctr;
        unsigned long long *dst[10] = {&w.p->stats->chunks_run, &w.p->stats->claim_misses, &w.p->stats->bytes_moved,
                                       &w.p->stats->busy_ns, &w.p->stats->inline_runs, &w.p->stats->slow_wrs,
                                       &w.p->stats->slow_issue_ns, &w.p->stats->job_slot_misses,
                                       &w.p->stats->publish_waits, &w.p->stats->publish_wait_ns};
        const unsigned long long val[10] = {c.n_chunks, c.n_miss, c.bytes, c.busy, c.n_inline,
                                            c.n_slow, c.t_slow, c.n_slot_miss, c.n_pub_wait, c.t_pub_wait};
#pragma unroll
        for (int i = 0; i < 10; ++i)
            if (val[i]) atomicAdd(dst[i], val[i]);
        c = WarpCounters{};
    }
    __syncwarp();
}

// ---- per-QP service ----------------------------------------------------------------------------

__device__ __forceinline__ uint4 ld_mr_part(const DevMr *m, int part) {
    return ld_vol128(reinterpret_cast<const uint8_t *>(m) + 16 * part);
}

// Validate and stage one WQE (in shared memory) into `rec`.  Warp-wide.  Every global load the
// checks need (local MRs by lane, the remote MR, the responder's configuration) is issued before
// any of them is used, so the whole validation costs one memory round trip.
// Warp-wide minimum / maximum of the lanes' values where `on` holds (~0 / 0 when none).
__device__ __forceinline__ uint64_t keep_lo(bool on, uint64_t v) {
    uint64_t a = on ? v : ~0ull;
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t t = __shfl_xor_sync(0xffffffffu, (unsigned long long)a, o);
        a = t < a ? t : a;
    }
    return a;
}
__device__ __forceinline__ uint64_t keep_hi(bool on, uint64_t v) {
    uint64_t a = on ? v : 0;
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t t = __shfl_xor_sync(0xffffffffu, (unsigned long long)a, o);
        a = t > a ? t : a;
    }
    return a;
}

__device__ __noinline__ void stage_wr(Warp &w, const QpView &v, const uint8_t *wqe, WrRec *rec, uint32_t *status_out,
                         uint64_t *total_out, uint64_t *remote_out, uint64_t *lo_out, uint64_t *hi_out) {
    const queue::SendWqe *h = reinterpret_cast<const queue::SendWqe *>(wqe);
    const uint32_t op = h->opcode;
    const uint32_t nsge = h->sge_count;
    uint32_t status = UGDR_WC_SUCCESS;
    const bool sum = op == UGDR_X_WR_RDMA_WRITE_SUM_BF16;
    const bool op_ok = op == UGDR_WR_RDMA_WRITE || op == UGDR_WR_RDMA_WRITE_WITH_IMM ||
                       op == UGDR_WR_RDMA_READ || is_atomic(op) || sum;
    if (!op_ok || nsge > v.max_sge || nsge > kMaxSge || (is_atomic(op) && nsge != 1))
        status = UGDR_WC_LOC_QP_OP_ERR;
    const bool mine = status == UGDR_WC_SUCCESS && uint32_t(w.lane) < nsge;
    const queue::Sge *sg = reinterpret_cast<const queue::Sge *>(wqe + queue::kSendSgeOffset) + (mine ? w.lane : 0);
    const uint64_t len = mine ? sg->length : 0;
    // --- issue every load ---
    uint4 l0{}, l1{}, l2{};
    if (mine && len != 0) {
        const DevMr *m = &w.p->mrs[(sg->lkey >> 1) & (kMaxMrs - 1)];
        l0 = ld_mr_part(m, 0);  // base, client_base
        l1 = ld_mr_part(m, 1);  // length, access, pd_num
        l2 = ld_mr_part(m, 2);  // lkey, rkey, valid, pad
    }
    const DevMr *rm = &w.p->mrs[(h->rkey >> 1) & (kMaxMrs - 1)];
    const uint4 r0 = ld_mr_part(rm, 0), r1 = ld_mr_part(rm, 1), r2 = ld_mr_part(rm, 2);
    uint32_t pstate = 0, perr = 0, pactive = 0, pacc = 0, ppd = 0;
    if (v.peer != nullptr) {
        pstate = ld_vol32(&v.peer->cfg.state);
        perr = ld_vol32(&v.peer->st.err);
        pactive = ld_vol32(&v.peer->cfg.active);
        pacc = ld_vol32(&v.peer->cfg.access);
        ppd = ld_vol32(&v.peer->cfg.pd_num);
    }
    // --- then check ---
    uint64_t local = 0;
    bool bad = false, lmc = false;
    if (mine && len != 0) {
        const uint64_t base = (uint64_t(l0.y) << 32) | l0.x, cb = (uint64_t(l0.w) << 32) | l0.z;
        const uint64_t ml = (uint64_t(l1.y) << 32) | l1.x;
        const uint32_t acc = l1.z, mpd = l1.w, lkey = l2.x, valid = l2.z;
        const bool need_write = op == UGDR_WR_RDMA_READ || is_atomic(op);
        if (!valid || lkey != sg->lkey || mpd != v.pd || base == 0 || sg->address < cb || len > ml ||
            sg->address - cb > ml - len || (need_write && (acc & UGDR_ACCESS_LOCAL_WRITE) == 0))
            bad = true;
        else
            local = base + (sg->address - cb);
        lmc = valid && (l2.w & kMrMulticast) != 0;
    }
    const bool any_bad = __any_sync(0xffffffffu, bad);
    uint64_t total = len;
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (status == UGDR_WC_SUCCESS && any_bad) status = UGDR_WC_LOC_PROT_ERR;
    if (status == UGDR_WC_SUCCESS && total > 0xffffffffull) status = UGDR_WC_LOC_LEN_ERR;  // 4 GiB - 1 max
    if (status == UGDR_WC_SUCCESS && is_atomic(op) && total != 8) status = UGDR_WC_LOC_LEN_ERR;
    // A multicast MR is only the single 16-byte aligned SGE of a WRITE_SUM_BF16.
    const bool any_lmc = __any_sync(0xffffffffu, lmc);
    if (status == UGDR_WC_SUCCESS && any_lmc &&
        (!sum || nsge != 1 || (__shfl_sync(0xffffffffu, (local | len), 0) & 15) != 0))
        status = UGDR_WC_LOC_QP_OP_ERR;
    if (status == UGDR_WC_SUCCESS && sum && nsge > 0) {
        // Every SGE has the same even length L, at a 2-byte aligned address; the WR moves L bytes.
        const uint64_t l0 = __shfl_sync(0xffffffffu, len, 0);
        const bool len_bad = mine && (len != l0 || (len & 1) != 0);
        const bool addr_bad = mine && (sg->address & 1) != 0;
        if (__any_sync(0xffffffffu, len_bad)) status = UGDR_WC_LOC_LEN_ERR;
        else if (__any_sync(0xffffffffu, addr_bad)) status = UGDR_WC_LOC_PROT_ERR;
        total = l0;
    }

    // Extent of the local segments (for the ordering rule).
    uint64_t lo = keep_lo(mine && len != 0 && !bad, local), hi = keep_hi(mine && len != 0 && !bad, local + len);
    // Compact the non-empty segments: lane i keeps slot = prefix count of non-empty lanes.
    const bool keep = mine && len != 0;
    const uint32_t keep_mask = __ballot_sync(0xffffffffu, keep);
    if (keep && status == UGDR_WC_SUCCESS) {
        const uint32_t idx = __popc(keep_mask & ((1u << w.lane) - 1));
        rec->seg[idx].local = local;
        rec->seg[idx].length = len;
    }

    uint64_t remote = 0;
    bool rmc = false;
    if (status == UGDR_WC_SUCCESS) {
        if (v.peer == nullptr || v.lost || pstate == UGDR_QPS_RESET || !pactive) {
            status = UGDR_WC_RETRY_EXC_ERR;
        } else if (pstate == UGDR_QPS_ERR || perr) {
            status = UGDR_WC_REM_OP_ERR;
        } else {
            const uint32_t need = remote_need(op);
            const uint64_t rlen = is_atomic(op) ? 8 : total;
            if ((pacc & need) == 0) {
                status = UGDR_WC_REM_ACCESS_ERR;
            } else if (rlen != 0) {
                const uint64_t base = (uint64_t(r0.y) << 32) | r0.x, cb = (uint64_t(r0.w) << 32) | r0.z;
                const uint64_t ml = (uint64_t(r1.y) << 32) | r1.x;
                const uint32_t acc = r1.z, mpd = r1.w, rkey = r2.y, valid = r2.z;
                const uint64_t ra = h->remote_address;
                if (!valid || rkey != h->rkey || mpd != ppd || base == 0 || (acc & need) == 0 || ra < cb ||
                    rlen > ml || ra - cb > ml - rlen)
                    status = UGDR_WC_REM_ACCESS_ERR;
                else
                    remote = base + (ra - cb);
                if (status == UGDR_WC_SUCCESS && is_atomic(op) && (ra & 7) != 0)
                    status = UGDR_WC_REM_INV_REQ_ERR;
                if (status == UGDR_WC_SUCCESS && sum && (ra & 1) != 0) status = UGDR_WC_REM_INV_REQ_ERR;
                rmc = valid && (r2.w & kMrMulticast) != 0;
                if (status == UGDR_WC_SUCCESS && rmc && (!sum || ((remote | total) & 15) != 0))
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
        rec->lo = lo < hi ? lo : 0;
        rec->hi = lo < hi ? hi : 0;
        rec->pad[0] = (any_lmc ? kWrSrcMulticast : 0u) | (rmc ? kWrDstMulticast : 0u);
    }
    __syncwarp();
    *status_out = status;
    *total_out = total;
    *remote_out = remote;
    *lo_out = lo < hi ? lo : 0;
    *hi_out = lo < hi ? hi : 0;
}

// Execute an inline WR (small payload or atomic) with the owner warp.  No fence here: the issue
// pass fences once for all the inline WRs it ran before any of them can retire.
__device__ void run_inline(Warp &w, WrRec *rec, const uint8_t *wqe, uint32_t op, uint64_t total,
                           uint64_t remote) {
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
        }
        __syncwarp();
        if (w.lane == 0) w.ctr->bytes += 8;
        return;
    }
    const uint32_t nseg = rec->nseg;
    if (op == UGDR_X_WR_RDMA_WRITE_SUM_BF16) {
        sum_stream(rec, nseg, remote, 0, total, w.lane);
    } else if (nseg == 1 && total <= 16 && op != UGDR_WR_RDMA_READ) {
        // Tiny payload: one lane per byte, no vector setup.
        const uint8_t *src = reinterpret_cast<const uint8_t *>(rec->seg[0].local);
        if (uint64_t(w.lane) < total) reinterpret_cast<uint8_t *>(remote)[w.lane] = src[w.lane];
    } else {
        copy_stream(rec, nseg, remote, op != UGDR_WR_RDMA_READ, 0, total, w.lane, nullptr);
    }
    __syncwarp();
    if (w.lane == 0) w.ctr->bytes += total;
}

// Retire finished WRs in order.  Lane i inspects WR head + i, so the ready prefix, the CQE list
// and its slot indices come out of one round of parallel loads and ballots; lane 0 then reserves
// and publishes every send CQE at once.  Returns WRs retired, or -1 / -2 on a wait that ran out.
// Commit the retirement of WRs [head, head + p): lane i (< p) holds WR head + i's completion
// fields.  Send CQEs go out with one reservation and one publish; the head then moves past every
// WR whose CQE found a slot.  Returns WRs retired (>= 0) or -1 when the publish wait ran out.
__device__ int retire_commit(Warp &w, DevQp *qp, const QpView &v, queue::Cqe *cqe_buf, uint64_t head, uint32_t p,
                             uint32_t err_mask, uint64_t wr_id, uint32_t status, uint32_t op, uint32_t signaled,
                             uint64_t total) {
    const uint64_t max_ns = w.p->max_wait_ns;
    int verdict = 0;
    const bool need = uint32_t(w.lane) < p && (signaled || status != UGDR_WC_SUCCESS);
    const uint32_t need_mask = __ballot_sync(0xffffffffu, need);
    if (need) {
        const uint32_t idx = __popc(need_mask & ((1u << w.lane) - 1));
        cqe_buf[idx] = queue::Cqe{wr_id, status, wc_op(op), status == UGDR_WC_SUCCESS ? uint32_t(total) : 0u, 0u,
                                  v.qpn, 0u};
    }
    __syncwarp();
    const uint32_t ncqe = __popc(need_mask);
    uint32_t retire_n = p;
    if (w.lane == 0) {
        uint32_t granted = 0;
        uint64_t first = 0;
        if (ncqe > 0) granted = reserve_cq(w, v.send_cq, ncqe, &first);
        w.t_reserved = gtime();
        if (granted < ncqe) {
            // Retire only the WRs before the first CQE that found no slot.
            uint32_t seen = 0;
            retire_n = 0;
            for (uint32_t i = 0; i < p; ++i) {
                const bool needs = (need_mask >> i) & 1u;
                if (needs && seen == granted) break;
                seen += needs ? 1u : 0u;
                ++retire_n;
            }
        }
        if (retire_n > 0) {
            // Return the SQ slots before the completions become visible: a client that polls a
            // CQE may post into its slot at once.  The WRs' fields are already in registers and
            // their payloads are done; the publish below is a release, so it orders this store.
            qp->st.sq_head = head + retire_n;
            st_vol64(&v.sq->head.value, head + retire_n);
        }
        if (granted > 0 && !publish_cq(w, v.send_cq, first, cqe_buf, granted, max_ns)) {
            verdict = -1;
        } else if (retire_n > 0) {
            atomicAdd(&w.p->stats->wrs_completed, (unsigned long long)retire_n);
            atomicAdd(&w.p->stats->retired, (unsigned long long)retire_n);
            atomicMax(&w.p->stats->last_end_ns, (unsigned long long)gtime());
            if (err_mask && retire_n == p) {
                atomicAdd(&w.p->stats->error_completions, 1ull);
                qp->st.errors += 1;
                qp->st.err = 1;
                st_rel_sys(&v.sq->meta.reserved[queue::kQpErrorWordIndex], UGDR_QPS_ERR);
            }
            verdict = int(retire_n);
        }
    }
    verdict = bcast(verdict);
    if (verdict > 0) {
        // Per-QP byte count: the successful WRs among the retired prefix, summed over the warp.
        unsigned long long b =
            uint32_t(w.lane) < uint32_t(verdict) && status == UGDR_WC_SUCCESS ? (unsigned long long)total : 0ull;
        for (int o = 16; o > 0; o >>= 1) b += __shfl_xor_sync(0xffffffffu, b, o);
        if (w.lane == 0) qp->st.bytes += b;
    }
    return verdict;
}

__device__ int retire(Warp &w, DevQp *qp, const QpView &v, queue::Cqe *cqe_buf) {
    const uint64_t max_ns = w.p->max_wait_ns;
    const uint64_t head = ld_vol(&qp->st.sq_head), issue = ld_vol(&qp->st.sq_issue);
    // The oldest batch's worth at most; a later pass retires the rest.
    const uint32_t m = issue - head < kBatch ? uint32_t(issue - head) : kBatch;
    if (m == 0) return 0;
    const bool mine = uint32_t(w.lane) < m;
    WrRec *rec = &qp->st.win[(head + (mine ? w.lane : 0)) % kWindow];
    uint32_t n = 0, done = 0, status = 0, op = 0, signaled = 0, recv_done = 0;
    unsigned long long wr_id = 0, total = 0;
    if (mine) {
        n = ld_vol32(&rec->nchunks);
        done = ld_vol32(&rec->chunks_done);
        status = ld_vol32(&rec->status);
        op = ld_vol32(&rec->opcode);
        signaled = ld_vol32(&rec->signaled);
        recv_done = ld_vol32(&rec->recv_cqe_done);
        wr_id = ld_vol(&rec->wr_id);
        total = ld_vol(&rec->total);
    }
    const uint32_t ready_mask = __ballot_sync(0xffffffffu, mine && (n == 0 || done >= n));
    uint32_t p = ones_prefix(ready_mask);  // ready prefix length
    if (p == 0) return 0;
    const uint32_t err_mask = __ballot_sync(0xffffffffu, uint32_t(w.lane) < p && status != UGDR_WC_SUCCESS);
    if (err_mask) p = __ffs(err_mask);  // retire up to and including the first error
    __threadfence();  // chunk workers' payload stores happen-before what follows
    // WRITE_WITH_IMM: responder completions first, in order, by lane 0.
    const uint32_t imm_mask = __ballot_sync(0xffffffffu, uint32_t(w.lane) < p && status == UGDR_WC_SUCCESS &&
                                                             op == UGDR_WR_RDMA_WRITE_WITH_IMM && !recv_done);
    int verdict = 0;
    if (imm_mask) {
        uint32_t stop = p;
        if (w.lane == 0) {
            for (uint32_t i = 0; i < p; ++i) {
                if (!(imm_mask & (1u << i))) continue;
                WrRec *r = &qp->st.win[(head + i) % kWindow];
                DevQp *peer = v.peer;
                if (peer != nullptr) {
                    DevCq *rcq = reinterpret_cast<DevCq *>(ld_vol(&peer->cfg.recv_cq));
                    const queue::Cqe rc{r->recv_wr_id, UGDR_WC_SUCCESS, UGDR_WC_RECV_RDMA_WITH_IMM,
                                        uint32_t(r->total), r->imm, ld_vol32(&peer->cfg.qpn), UGDR_WC_WITH_IMM};
                    const int prc = produce_cqe(w, rcq, rc, max_ns);
                    if (prc == 1) {  // responder CQ full: retry on a later pass
                        stop = i;
                        break;
                    }
                    if (prc == 2 || !release_rq(peer, r->recv_claim, max_ns)) {
                        verdict = prc == 2 ? -1 : -2;
                        stop = i;
                        break;
                    }
                }
                r->recv_cqe_done = 1;
            }
        }
        verdict = bcast(verdict);
        if (verdict < 0) return verdict;
        p = bcast(stop);
        if (p == 0) return 0;
    }
    return retire_commit(w, qp, v, cqe_buf, head, p, err_mask, wr_id, status, op, signaled, total);
}

// Lane-parallel issue: lane j validates WQE j of the staged batch (single-SGE WRITE / READ of
// any size), so a batch costs one round of parallel loads instead of one round trip per WR.
// Payloads of at most kLaneBytes are copied by their lane on the spot; larger ones become one
// chunked job for the whole batch (chunks numbered across its WRs), which every warp of the GPU
// may claim.  Processes the longest prefix of such WQEs and returns its length (an erroring WQE
// ends the prefix and is included; nothing after it runs).  *chunked_out tells whether any WR
// of the prefix went to a job (then it completes later, through retire()).
constexpr uint32_t kLaneBytes = 64;

// Chunk size for a job whose largest WR is `max_len`: about half the warps get a chunk of a
// lone WR, within [kChunkMin, kChunkMax], so claims stay rare next to the copies.
__device__ __forceinline__ uint32_t chunk_for(uint64_t max_len, uint32_t nwarps) {
    const uint64_t cb = max_len / (nwarps / 2 + 1);
    uint32_t chunk = kChunkMin;
    while (chunk < cb && chunk < kChunkMax) chunk <<= 1;
    return chunk;
}

struct LaneWr {
    uint64_t wr_id, total;
    uint32_t status, op, signaled;
};

__device__ uint32_t issue_fast(Warp &w, DevQp *qp, const QpView &v, const uint8_t *wqe_smem, uint32_t st, uint64_t head,
                               uint64_t issue0, uint32_t avail, LaneWr *out, JobRing *jr, uint32_t *bitmap,
                               uint32_t nwarps, bool *chunked_out) {
    *chunked_out = false;
    const uint32_t j = uint32_t(w.lane);
    const bool in = j < avail;
    const queue::SendWqe *h = reinterpret_cast<const queue::SendWqe *>(wqe_smem + (in ? j : 0) * st);
    const queue::Sge *sg = reinterpret_cast<const queue::Sge *>(wqe_smem + (in ? j : 0) * st +
                                                                queue::kSendSgeOffset);
    const uint32_t op = h->opcode;
    const bool fast = in && (op == UGDR_WR_RDMA_WRITE || op == UGDR_WR_RDMA_READ) && h->sge_count == 1 &&
                      sg->length <= 0x80000000u && v.max_sge >= 1;
    const uint32_t fast_mask = __ballot_sync(0xffffffffu, fast);
    const uint32_t p = ones_prefix(fast_mask);
    if (p == 0) return 0;
    const bool act = j < p;
    const uint64_t len = act ? sg->length : 0;
    // --- MR entries (warp cache, else one parallel round of loads); responder config from the
    // QP view ---
    uint4 l0{}, l1{}, l2{}, r0{}, r1{}, r2{};
    const MrCacheEntry *lc = &w.mrc[0], *rc = &w.mrc[1];
    const bool lhit = act && lc->key == sg->lkey && sg->lkey != 0 && lc->epoch == w.epoch;
    const bool rhit = act && rc->key == h->rkey && h->rkey != 0 && rc->epoch == w.epoch;
    if (act) {
        if (lhit) {
            l0 = lc->part[0];
            l1 = lc->part[1];
            l2 = lc->part[2];
        } else {
            const DevMr *lm = &w.p->mrs[(sg->lkey >> 1) & (kMaxMrs - 1)];
            l0 = ld_mr_part(lm, 0);
            l1 = ld_mr_part(lm, 1);
            l2 = ld_mr_part(lm, 2);
        }
        if (rhit) {
            r0 = rc->part[0];
            r1 = rc->part[1];
            r2 = rc->part[2];
        } else {
            const DevMr *rm = &w.p->mrs[(h->rkey >> 1) & (kMaxMrs - 1)];
            r0 = ld_mr_part(rm, 0);
            r1 = ld_mr_part(rm, 1);
            r2 = ld_mr_part(rm, 2);
        }
    }
    __syncwarp();
    if (j == 0 && act) {  // remember lane 0's entries (only valid ones)
        if (!lhit && l2.z && l2.x == sg->lkey) {
            w.mrc[0].key = sg->lkey;
            w.mrc[0].epoch = w.epoch;
            w.mrc[0].part[0] = l0;
            w.mrc[0].part[1] = l1;
            w.mrc[0].part[2] = l2;
        }
        if (!rhit && r2.z && r2.y == h->rkey) {
            w.mrc[1].key = h->rkey;
            w.mrc[1].epoch = w.epoch;
            w.mrc[1].part[0] = r0;
            w.mrc[1].part[1] = r1;
            w.mrc[1].part[2] = r2;
        }
    }
    __syncwarp();
    const uint32_t pstate = v.pstate, perr = v.perr, pactive = v.pactive, pacc = v.pacc, ppd = v.ppd;
    // --- check ---
    uint32_t status = UGDR_WC_SUCCESS;
    uint64_t local = 0, remote = 0;
    if (act && len != 0 && ((l2.w | r2.w) & kMrMulticast) != 0) {
        // Multicast views serve WRITE_SUM_BF16 only.
        status = (l2.w & kMrMulticast) ? UGDR_WC_LOC_QP_OP_ERR : UGDR_WC_REM_INV_REQ_ERR;
    } else if (act && len != 0) {
        const uint64_t base = (uint64_t(l0.y) << 32) | l0.x, cb = (uint64_t(l0.w) << 32) | l0.z;
        const uint64_t ml = (uint64_t(l1.y) << 32) | l1.x;
        const bool need_write = op == UGDR_WR_RDMA_READ;
        if (!l2.z || l2.x != sg->lkey || l1.w != v.pd || base == 0 || sg->address < cb || len > ml ||
            sg->address - cb > ml - len || (need_write && (l1.z & UGDR_ACCESS_LOCAL_WRITE) == 0))
            status = UGDR_WC_LOC_PROT_ERR;
        else
            local = base + (sg->address - cb);
    }
    if (act && status == UGDR_WC_SUCCESS) {
        if (v.peer == nullptr || v.lost || pstate == UGDR_QPS_RESET || !pactive) {
            status = UGDR_WC_RETRY_EXC_ERR;
        } else if (pstate == UGDR_QPS_ERR || perr) {
            status = UGDR_WC_REM_OP_ERR;
        } else {
            const uint32_t need = remote_need(op);
            if ((pacc & need) == 0) {
                status = UGDR_WC_REM_ACCESS_ERR;
            } else if (len != 0) {
                const uint64_t base = (uint64_t(r0.y) << 32) | r0.x, cb = (uint64_t(r0.w) << 32) | r0.z;
                const uint64_t ml = (uint64_t(r1.y) << 32) | r1.x;
                const uint64_t ra = h->remote_address;
                if (!r2.z || r2.y != h->rkey || r1.w != ppd || base == 0 || (r1.z & need) == 0 || ra < cb ||
                    len > ml || ra - cb > ml - len)
                    status = UGDR_WC_REM_ACCESS_ERR;
                else
                    remote = base + (ra - cb);
            }
        }
    }
    const uint32_t err_mask = __ballot_sync(0xffffffffu, act && status != UGDR_WC_SUCCESS);
    uint32_t count = err_mask ? __ffs(err_mask) : p;  // through the first error, inclusive
    // --- ordering: stop before the first WR that touches bytes an earlier one may still move ---
    {
        const Span sp = span_of(op, remote, len, local, local + len, j < count && status == UGDR_WC_SUCCESS && len != 0);
        const bool c = clashes_in_batch(w, count, sp);
        const bool f = clashes_in_flight(w, qp, head, issue0, sp);
        const uint32_t clash_mask = __ballot_sync(0xffffffffu, j < count && (c || f));
        if (clash_mask) {
            if (w.lane == 0) atomicAdd(&w.p->stats->order_waits, 1ull);
            count = __ffs(clash_mask) - 1;
            if (count == 0) return 0;
        }
    }
    // --- chunked WRs: one job for the batch; its slot is taken before anything runs ---
    bool chunked = j < count && status == UGDR_WC_SUCCESS && len > kLaneBytes;
    uint32_t chunk_mask = __ballot_sync(0xffffffffu, chunked);
    int slot = -1;
    unsigned long long gen = 0;
    uint32_t cb = 0;
    if (chunk_mask) {
        if (w.lane == 0) slot = take_job_slot(jr, w.gwarp + uint32_t(issue0), &gen);
        slot = bcast(slot);
        if (slot < 0) {
            // No free slot: only the WRs before the first chunked one run now.
            if (w.lane == 0) w.ctr->n_slot_miss += 1;
            count = __ffs(chunk_mask) - 1;
            chunk_mask = 0;
            chunked = false;
            if (count == 0) return 0;
        } else {
            gen = bcast64(gen);
            uint64_t mx = chunked ? len : 0;
            for (int o = 16; o > 0; o >>= 1) {
                const uint64_t t = __shfl_xor_sync(0xffffffffu, mx, o);
                mx = t > mx ? t : mx;
            }
            cb = chunk_for(mx, nwarps);
        }
    }
    const uint32_t nch = chunked ? uint32_t((len + cb - 1) / cb) : 0u;
    uint32_t start = nch;  // inclusive scan, then made exclusive
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, start, o);
        if (w.lane >= o) start += t;
    }
    const uint32_t total_chunks = __shfl_sync(0xffffffffu, start, 31);
    start -= nch;
    // --- execute (lanes before the first error only) ---
    if (j < count && !chunked && status == UGDR_WC_SUCCESS && len != 0) {
        uint8_t *dst = reinterpret_cast<uint8_t *>(op == UGDR_WR_RDMA_READ ? local : remote);
        const uint8_t *src = reinterpret_cast<const uint8_t *>(op == UGDR_WR_RDMA_READ ? remote : local);
        if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | len) & 7) == 0) {
            for (uint64_t o = 0; o < len; o += 8)
                *reinterpret_cast<uint64_t *>(dst + o) = *reinterpret_cast<const uint64_t *>(src + o);
        } else {
            for (uint64_t o = 0; o < len; ++o) dst[o] = src[o];
        }
    }
    uint64_t lane_bytes = 0;
    if (j < count) {
        WrRec *rec = &qp->st.win[(issue0 + j) % kWindow];
        rec->wr_id = h->wr_id;
        rec->opcode = op;
        rec->total = len;
        rec->remote = remote;
        rec->status = status;
        rec->imm = 0;
        rec->nseg = len != 0 ? 1 : 0;
        rec->seg[0].local = local;
        rec->seg[0].length = len;
        rec->lo = len != 0 ? local : 0;
        rec->hi = len != 0 ? local + len : 0;
        rec->recv_cqe_done = 0;
        rec->chunks_done = 0;
        rec->nchunks = nch;
        rec->signaled = (v.sig_all || (h->send_flags & UGDR_SEND_SIGNALED) != 0) ? 1u : 0u;
        lane_bytes = chunked ? 0 : len;
        *out = LaneWr{h->wr_id, len, status, op, rec->signaled};
    }
    __syncwarp();
    for (int o = 16; o > 0; o >>= 1) lane_bytes += __shfl_xor_sync(0xffffffffu, lane_bytes, o);
    if (w.lane == 0) w.ctr->bytes += lane_bytes;
    if (chunk_mask) {
        publish_job(w, jr, bitmap, slot, gen, qp->st.win, uint32_t(issue0 % kWindow), count, start, total_chunks, cb);
        *chunked_out = true;
    }
    return count;
}

__device__ uint32_t service_cached(Warp &w, DevQp *qp, QpView &v, uint8_t *wqe_smem, queue::Cqe *cqe_smem,
                                   JobRing *jr, uint32_t *bitmap, uint32_t nwarps);

// Service one QP: retire, flush when in ERR, else issue a batch of WQEs and retire again.
// Warp-wide; returns the work done.
__device__ uint32_t service_pass(Warp &w, DevQp *qp, uint8_t *wqe_smem, queue::Cqe *cqe_smem, JobRing *jr,
                                 uint32_t *bitmap, uint32_t nwarps);

// One service pass over a QP under the current MR epoch, then its progress record (see
// QpProgress): the epoch the pass started with and the cursors after it.
__device__ uint32_t service_qp(Warp &w, DevQp *qp, uint8_t *wqe_smem, queue::Cqe *cqe_smem, JobRing *jr,
                               uint32_t *bitmap, uint32_t nwarps) {
    w.epoch = *w.mr_epoch;
    __syncwarp();
    const uint32_t work = service_pass(w, qp, wqe_smem, cqe_smem, jr, bitmap, nwarps);
    if (w.lane == 0 && w.vq == qp) {
        QpProgress *pr = &w.p->progress[qp - w.p->qps];
        st_vol64(&pr->epoch_issue, (uint64_t(w.epoch) << 32) | (w.vissue & 0xffffffffull));
        st_vol64(&pr->head, w.vhead);
    }
    return work;
}

__device__ uint32_t service_pass(Warp &w, DevQp *qp, uint8_t *wqe_smem, queue::Cqe *cqe_smem, JobRing *jr,
                                 uint32_t *bitmap, uint32_t nwarps) {
    const uint64_t max_ns = w.p->max_wait_ns;
    // The configuration this pass needs: cached per warp for the QP it serviced last and re-read
    // at least every 20 us, and at once under a new MR epoch: the host bumps the epoch and waits
    // for every QP's next pass when a change must be seen by a deadline (a peer unbound before
    // its QP goes away).  The owner warp is the only writer of the QP's cursors, so the cached
    // head / issue are authoritative.
    const uint64_t now0 = gtime();
    if (w.vq == qp && now0 - w.vt < 20000 && w.vepoch == w.epoch) {
        return service_cached(w, qp, *w.vv, wqe_smem, cqe_smem, jr, bitmap, nwarps);
    }
    if (!ld_vol32(&qp->cfg.active)) {
        w.vq = nullptr;
        return 0;
    }
    QpView v;
    v.sq = reinterpret_cast<queue::RingHeader *>(ld_vol(&qp->cfg.sq));
    v.sq_slots = reinterpret_cast<const uint8_t *>(ld_vol(&qp->cfg.sq_slots));
    v.peer = reinterpret_cast<DevQp *>(ld_vol(&qp->cfg.peer));
    v.send_cq = reinterpret_cast<DevCq *>(ld_vol(&qp->cfg.send_cq));
    v.sq_cap = ld_vol32(&qp->cfg.sq_cap);
    v.sq_stride = ld_vol32(&qp->cfg.sq_stride);
    v.qpn = ld_vol32(&qp->cfg.qpn);
    v.state = ld_vol32(&qp->cfg.state);
    v.pd = ld_vol32(&qp->cfg.pd_num);
    v.max_sge = ld_vol32(&qp->cfg.max_send_sge);
    v.sig_all = ld_vol32(&qp->cfg.sq_sig_all);
    v.lost = ld_vol32(&qp->cfg.peer_lost);
    v.err = ld_vol32(&qp->st.err);
    v.err_issued = ld_vol32(&qp->st.err_issued);
    v.retry_word = ld_vol32(&qp->cfg.timeout);  // timeout, retry_cnt, rnr_retry, min_rnr_timer
    v.pstate = v.perr = v.pactive = v.pacc = v.ppd = 0;
    if (v.peer != nullptr) {
        v.pstate = ld_vol32(&v.peer->cfg.state);
        v.perr = ld_vol32(&v.peer->st.err);
        v.pactive = ld_vol32(&v.peer->cfg.active);
        v.pacc = ld_vol32(&v.peer->cfg.access);
        v.ppd = ld_vol32(&v.peer->cfg.pd_num);
    }
    w.vhead = ld_vol(&qp->st.sq_head);
    w.vissue = ld_vol(&qp->st.sq_issue);
    w.vtail = w.vissue;
    w.vq = qp;
    __syncwarp();
    if (w.lane == 0) *w.vv = v;
    __syncwarp();
    w.vt = now0;
    w.vepoch = w.epoch;
    return service_cached(w, qp, *w.vv, wqe_smem, cqe_smem, jr, bitmap, nwarps);
}

// An error WR was issued: later passes issue nothing on this QP until it retires and the QP
// enters ERR (whose flush then completes every WR behind it).
__device__ void mark_err_issued(Warp &w, DevQp *qp, QpView &v) {
    __syncwarp();
    if (w.lane == 0) {
        *reinterpret_cast<volatile uint32_t *>(&qp->st.err_issued) = 1u;
        v.err_issued = 1;
    }
    __syncwarp();
}

__device__ uint32_t service_cached(Warp &w, DevQp *qp, QpView &v, uint8_t *wqe_smem, queue::Cqe *cqe_smem,
                                   JobRing *jr, uint32_t *bitmap, uint32_t nwarps) {
    const uint64_t max_ns = w.p->max_wait_ns;
    uint32_t work = 0;

    int r = 0;
    if (w.vhead != w.vissue) {
        const uint64_t t_r0 = gtime();
        r = retire(w, qp, v, cqe_smem);
        if (r > 0 && w.lane == 0 && w.p->trace != nullptr)
            trace_event(w.p, kTraceRetire, w.gwarp, uint32_t(qp - w.p->qps), uint32_t(r), t_r0, gtime());
        if (r < 0) {
            record_error(w, r == -1 ? kErrCqPublishTimeout : kErrRqReleaseTimeout);
            return work;
        }
        w.vhead += uint64_t(r);
        work += uint32_t(r);
        if (r > 0 && ld_vol32(&qp->st.err) != 0) v.err = 1;
    }

    const bool in_error = v.state == UGDR_QPS_ERR || v.err != 0;
    if (in_error) {
        // Flush once nothing is in flight: every unissued SQ WR and every posted RQ WR.
        int flushed = 0;
        if (w.lane == 0 && qp->st.sq_head == qp->st.sq_issue) {
            DevCq *rcq = reinterpret_cast<DevCq *>(ld_vol(&qp->cfg.recv_cq));
            const uint64_t tail = ld_acq_sys(&v.sq->tail.value);
            while (qp->st.sq_issue < tail && flushed >= 0) {
                const uint8_t *slot = v.sq_slots + (qp->st.sq_issue % v.sq_cap) * v.sq_stride;
                const uint64_t wr_id = ld_vol(slot);
                const uint32_t op = ld_vol32(slot + 20);
                const queue::Cqe c{wr_id, UGDR_WC_WR_FLUSH_ERR, wc_op(op), 0u, 0u, v.qpn, 0u};
                const int prc = produce_cqe(w, v.send_cq, c, max_ns);
                if (prc == 1) break;
                if (prc == 2) {
                    flushed = -1;
                    break;
                }
                qp->st.sq_issue += 1;
                qp->st.sq_head = qp->st.sq_issue;
                st_rel_sys(&v.sq->head.value, qp->st.sq_head);
                atomicAdd(&w.p->stats->error_completions, 1ull);
                qp->st.errors += 1;
                atomicAdd(&w.p->stats->retired, 1ull);
                ++flushed;
            }
            uint64_t claim = 0, wr_id = 0;
            while (flushed >= 0 && claim_rq(qp, &claim, &wr_id)) {
                const queue::Cqe c{wr_id, UGDR_WC_WR_FLUSH_ERR, UGDR_WC_RECV_RDMA_WITH_IMM, 0u, 0u, v.qpn, 0u};
                // Receive CQ full: wait (bounded) for the consumer; the claim is already taken.
                int prc;
                const uint64_t t0 = gtime();
                while ((prc = produce_cqe(w, rcq, c, max_ns)) == 1 && gtime() - t0 < max_ns) __nanosleep(256);
                if (prc != 0 || !release_rq(qp, claim, max_ns)) {
                    flushed = -2;
                    break;
                }
                atomicAdd(&w.p->stats->error_completions, 1ull);
                qp->st.errors += 1;
                ++flushed;
            }
        }
        flushed = bcast(flushed);
        if (flushed < 0) record_error(w, flushed == -1 ? kErrCqPublishTimeout : kErrRqReleaseTimeout);
        w.vhead = ld_vol(&qp->st.sq_head);
        w.vissue = ld_vol(&qp->st.sq_issue);
        return work + (flushed > 0 ? flushed : 0);
    }
    if (v.state != UGDR_QPS_RTS || v.err_issued) return work;  // an error WR in flight: wait for its retire

    // Issue: one lane-parallel fetch of every WQE that fits the window and the staging buffer.
    // The SQ tail (a PCIe read) is read only when the window has room and the tail seen last
    // does not already cover it: WQEs below a tail acquired earlier are as valid now.
    // On a queue whose slots are wider than 64 B (max_send_sge > 1) only each slot's first 64 B
    // are fetched at first: a WQE of at most one SGE (atomics included) lies wholly inside them,
    // so up to kWqeStage / 64 such WQEs are staged per pass, as on a one-SGE queue.  The batch
    // ends before the first wider WQE; when that is the first one, the pass fetches as many
    // whole slots as the staging buffer holds.
    const uint64_t head = w.vhead, issue0 = w.vissue;
    const uint32_t wide = v.sq_stride > 64 ? 1u : 0u;
    uint32_t st = wide ? 64u : v.sq_stride;  // stage stride: bytes per staged WQE
    uint64_t room = kWindow - (issue0 - head);
    if (room > kWqeStage / st) room = kWqeStage / st;
    if (room == 0) return work;
    if (w.vtail < issue0 + room) {
        uint64_t tail = 0;
        if (w.lane == 0) tail = ld_acq_sys(&v.sq->tail.value);
        w.vtail = bcast64(tail);
    }
    const uint64_t tail = w.vtail;
    uint64_t avail = tail > issue0 ? tail - issue0 : 0;
    if (avail > room) avail = room;
    if (avail == 0) return work;
    const uint64_t t_fetch0 = gtime();
    const uint32_t nbytes = uint32_t(avail) * st;
    for (uint32_t o = w.lane * 16; o < nbytes; o += 32 * 16) {
        const uint64_t s = issue0 + o / st;
        const uint8_t *src = v.sq_slots + (s % v.sq_cap) * v.sq_stride + (o % st);
        *reinterpret_cast<uint4 *>(wqe_smem + o) = ld_vol128(src);
    }
    __syncwarp();
    if (wide) {
        const bool in = uint32_t(w.lane) < avail;
        const uint32_t nsge = in ? reinterpret_cast<const queue::SendWqe *>(wqe_smem + w.lane * 64)->sge_count : 0;
        const uint32_t narrow = __ballot_sync(0xffffffffu, in && nsge <= 1);
        const uint32_t p = ones_prefix(narrow);  // WQEs before the first wide one
        __syncwarp();
        if (p > 0) {
            avail = p;
        } else {  // the first WQE is wide: as many as fit, in full
            const uint64_t fit = kWqeStage / v.sq_stride;
            avail = avail < fit ? avail : fit;
            st = v.sq_stride;
            const uint32_t nb = uint32_t(avail) * st;
            for (uint32_t o = w.lane * 16; o < nb; o += 32 * 16) {
                const uint64_t s = issue0 + o / st;
                *reinterpret_cast<uint4 *>(wqe_smem + o) = ld_vol128(v.sq_slots + (s % v.sq_cap) * st + (o % st));
            }
            __syncwarp();
        }
    }
    uint32_t inline_ran = 0;
    const uint64_t t_fetch1 = gtime();
    LaneWr lw{0, 0, 0, 0, 0};
    bool fast_chunked = false;
    uint64_t issued = issue_fast(w, qp, v, wqe_smem, st, head, issue0, uint32_t(avail), &lw, jr, bitmap, nwarps,
                                 &fast_chunked);
    const uint32_t fast_n = uint32_t(issued);
    if (w.lane == 0 && w.p->trace != nullptr) {
        // Issue pass: WRs issued by the fast path | in flight before << 8 | fetched << 16 |
        // unissued WQEs seen (capped) << 24.
        const uint64_t seen = tail - issue0 < 255 ? tail - issue0 : 255;
        trace_event(w.p, kTraceIssue, w.gwarp, uint32_t(qp - w.p->qps),
                    fast_n | uint32_t(issue0 - head) << 8 | uint32_t(avail) << 16 | uint32_t(seen) << 24, t_fetch0,
                    gtime());
    }
    if (issued > 0) {
        if (w.lane == 0 && head != issue0) atomicAdd(&w.p->stats->overlap_issues, 1ull);
        inline_ran += uint32_t(issued);
        if (w.lane == 0 && !w.started) atomicCAS(&w.p->stats->first_start_ns, 0ull, (unsigned long long)gtime());
        w.started = true;
    }
    const uint32_t fast_err = __ballot_sync(0xffffffffu, uint32_t(w.lane) < fast_n && lw.status != 0);
    if (fast_err) mark_err_issued(w, qp, v);
    // Staged WRs that need chunk copies share ONE job: the first takes the slot, each adds its
    // chunks (lane i holds WR i's first chunk index), staged inline WRs after it join with zero
    // chunks so the job's WRs stay consecutive in the window, and the job is published once,
    // when the loop ends for whatever reason.
    int bslot = -1;
    unsigned long long bgen = 0;
    uint32_t bfirst = 0, bn = 0, bchunks = 0, bcb = 0, my_start = 0;
    for (uint64_t j = fast_err ? avail : issued; j < avail; ++j) {
        const uint64_t issue = issue0 + j;
        const uint8_t *wqe = wqe_smem + j * st;
        WrRec *rec = &qp->st.win[issue % kWindow];
        uint32_t status;
        uint64_t total, remote, lo, hi;
        const uint64_t t_stage = gtime();
        stage_wr(w, v, wqe, rec, &status, &total, &remote, &lo, &hi);
        const queue::SendWqe *h = reinterpret_cast<const queue::SendWqe *>(wqe);
        const uint32_t op = h->opcode;
        const bool signaled = v.sig_all || (h->send_flags & UGDR_SEND_SIGNALED) != 0;
        // Ordering: wait (a later pass) while an earlier WR still in flight touches its bytes.
        if (__any_sync(0xffffffffu,
                       clashes_in_flight(w, qp, head, issue,
                                         span_of(op, remote, total, lo, hi, status == UGDR_WC_SUCCESS)))) {
            if (w.lane == 0) atomicAdd(&w.p->stats->order_waits, 1ull);
            break;
        }

        // A WR that becomes a job takes its job slot first: with no slot free the WR waits for a
        // later pass before anything (an RQ claim, a copy) has been done for it.
        const bool needs_job = status == UGDR_WC_SUCCESS && !is_atomic(op) && total > kInlineBytes;
        bool took = false;  // this WR took the batch's job slot
        if (needs_job && bslot < 0) {
            int slot = -1;
            unsigned long long gen = 0;
            if (w.lane == 0) slot = take_job_slot(jr, w.gwarp + uint32_t(issue), &gen);
            slot = bcast(slot);
            if (slot < 0) {  // no job slot: retry on a later pass
                if (w.lane == 0) w.ctr->n_slot_miss += 1;
                break;
            }
            bslot = slot;
            bgen = bcast64(gen);
            took = true;
        }

        // Responder RQ for WRITE_WITH_IMM (RNR when empty).
        int rnr = 0;  // 0 go, 1 wait, 2 retry budget exhausted
        if (status == UGDR_WC_SUCCESS && op == UGDR_WR_RDMA_WRITE_WITH_IMM) {
            if (w.lane == 0) {
                uint64_t claim = 0, wr_id = 0;
                if (claim_rq(v.peer, &claim, &wr_id)) {
                    rec->recv_claim = claim;
                    rec->recv_wr_id = wr_id;
                    qp->st.rnr_attempts = 0;
                    qp->st.rnr_next_ns = 0;
                } else {
                    const uint8_t rnr_retry = uint8_t(v.retry_word >> 16);
                    if (rnr_retry == 7) {
                        rnr = 1;
                    } else {
                        const uint64_t now = gtime();
                        if (qp->st.rnr_next_ns == 0 || now >= qp->st.rnr_next_ns) {
                            if (qp->st.rnr_next_ns != 0) qp->st.rnr_attempts += 1;
                            if (qp->st.rnr_attempts >= rnr_retry) {
                                rnr = 2;
                            } else {
                                const uint32_t code = ld_vol32(&v.peer->cfg.timeout) >> 24;
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
            if (rnr != 0 && took) {
                // No job after all: hand the taken slot back (its sequence becomes even again).
                if (w.lane == 0) atomicAdd(&jr->slots[bslot].seq, 1ull);
                bslot = -1;
            }
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
            if (!w.started) atomicCAS(&w.p->stats->first_start_ns, 0ull, (unsigned long long)gtime());
        }
        w.started = true;
        if (status == UGDR_WC_SUCCESS) {
            if (!(needs_job && bslot >= 0)) {
                run_inline(w, rec, wqe, op, total, remote);
                ++inline_ran;
                if (bn > 0) {  // inside the job's range, with no chunks
                    if (uint32_t(w.lane) == bn) my_start = bchunks;
                    ++bn;
                }
            } else {
                if (bn == 0) {
                    bfirst = uint32_t(issue % kWindow);
                    bcb = chunk_for(total, nwarps);
                }
                const uint32_t n = uint32_t((total + bcb - 1) / bcb);
                if (w.lane == 0) rec->nchunks = n;
                if (uint32_t(w.lane) == bn) my_start = bchunks;
                ++bn;
                bchunks += n;
            }
        }
        if (w.lane == 0) w.ctr->n_slow += 1;
        if (w.lane == 0) w.ctr->t_slow += gtime() - t_stage;
        ++issued;
        if (status != UGDR_WC_SUCCESS) {  // stop issuing behind an error
            mark_err_issued(w, qp, v);
            break;
        }
    }
    if (bslot >= 0) {
        if (bchunks > 0) {
            __syncwarp();
            publish_job(w, jr, bitmap, bslot, bgen, qp->st.win, bfirst, bn, my_start, bchunks, bcb);
        } else if (w.lane == 0) {
            atomicAdd(&jr->slots[bslot].seq, 1ull);  // nothing to copy after all: free the slot
        }
    }
    if (issued > 0) {
        __syncwarp();
        if (w.lane == 0) {
            // No fence: the issue cursor is private to this warp, and the publish path's system
            // fence orders these inline payload stores before any of their CQEs.
            qp->st.sq_issue = issue0 + issued;
        }
        __syncwarp();
        w.vissue = issue0 + issued;
        if (w.lane == 0) w.ctr->n_inline += inline_ran;
        work += uint32_t(issued);
        if (head == issue0 && issued == fast_n && !fast_chunked) {
            // Only this fast batch is in flight and every lane still holds its WR: retire it
            // without reading anything back.
            const uint32_t err_mask = __ballot_sync(0xffffffffu, uint32_t(w.lane) < fast_n && lw.status != 0);
            const uint64_t t_exec1 = gtime();
            r = retire_commit(w, qp, v, cqe_smem, head, fast_n, err_mask, lw.wr_id, lw.status, lw.op, lw.signaled,
                              lw.total);
            if (w.lane == 0) {
                const uint64_t t_end = gtime();
                const uint64_t t_res = w.t_reserved > t_exec1 ? w.t_reserved : t_exec1;
                atomicAdd(&w.p->stats->fast_batches, 1ull);
                atomicAdd(&w.p->stats->fast_fetch_ns, (unsigned long long)(t_fetch1 - t_fetch0));
                atomicAdd(&w.p->stats->fast_exec_ns, (unsigned long long)(t_exec1 - t_fetch1));
                atomicAdd(&w.p->stats->fast_reserve_ns, (unsigned long long)(t_res - t_exec1));
                atomicAdd(&w.p->stats->fast_publish_ns, (unsigned long long)(t_end - t_res));
                if (w.p->trace != nullptr)
                    trace_event(w.p, kTraceFastBatch, w.gwarp, uint32_t(qp - w.p->qps), fast_n, t_fetch0, t_end);
            }
        } else {
            const uint64_t t_r0 = gtime();
            r = retire(w, qp, v, cqe_smem);
            if (r > 0 && w.lane == 0 && w.p->trace != nullptr)
                trace_event(w.p, kTraceRetire, w.gwarp, uint32_t(qp - w.p->qps), uint32_t(r), t_r0, gtime());
        }
        if (r < 0) {
            record_error(w, r == -1 ? kErrCqPublishTimeout : kErrRqReleaseTimeout);
            return work;
        }
        w.vhead += uint64_t(r);
        work += uint32_t(r);
        if (r > 0 && ld_vol32(&qp->st.err) != 0) v.err = 1;
    }
    return work;
}

// Warp 0 of every CTA is its leader: it services its own QPs and, about every microsecond,
// mirrors the global control words (job bitmap, QP-slot bound, exit / stop / drain state) into
// shared memory.  The other warps service their QPs and copy chunks, reading only the mirror when
// idle.  Without the mirror every warp of the grid polled the same few L2 lines and every
// data access hashing to those slices queued behind the polls.
__global__ void __launch_bounds__(kThreads, 1) executor_kernel(ExecParams p) {
    extern __shared__ __align__(128) uint8_t tma_smem[];  // (kWarps - 1) x kTmaStages x kTmaPiece
    __shared__ __align__(8) uint64_t tma_bar[kWarps][kTmaStages];
    __shared__ Tma tma_state[kWarps];
    __shared__ __align__(16) uint8_t wqe_buf[kWarps][kWqeStage];
    __shared__ __align__(16) queue::Cqe cqe_buf[kWarps][kBatch];
    __shared__ __align__(16) MrCacheEntry mr_cache[kWarps][2];
    __shared__ WarpCounters counters[kWarps];
    __shared__ CqCache cq_cache[kWarps];
    __shared__ QpView qp_view[kWarps];
    __shared__ volatile uint32_t s_bits[32];
    __shared__ volatile uint32_t s_slots, s_exit, s_work, s_epoch;
    Warp w;
    w.p = &p;
    w.lane = threadIdx.x & 31;
    w.wi = threadIdx.x >> 5;
    w.gwarp = blockIdx.x * kWarps + w.wi;
    w.rot = w.gwarp * 2654435761u;
    w.abort = false;
    w.ctr = &counters[w.wi];
    if (w.lane == 0) counters[w.wi] = WarpCounters{};
    w.started = false;
    w.cq = &cq_cache[w.wi];
    w.vv = &qp_view[w.wi];
    if (w.lane == 0) w.cq->cq = nullptr;
    w.vq = nullptr;
    w.vepoch = 0;
    w.mrc = mr_cache[w.wi];
    w.mirror = s_bits;
    if (w.lane < 2) w.mrc[w.lane].key = 0;
    w.tma = nullptr;
    if (w.wi != 0) {  // chunk workers: TMA staging and its barriers, fresh for every launch
        w.tma = &tma_state[w.wi];
        if (w.lane == 0) {
            Tma &t = tma_state[w.wi];
            t.buf = tma_smem + size_t(w.wi - 1) * kTmaStages * kTmaPiece;
            t.bar = tma_bar[w.wi];
            t.phase = 0;
            t.min = !kTmaBuilt ? 0u : p.bulk_min < kTmaPiece && p.bulk_min != 0 ? kTmaPiece : p.bulk_min;
            t.failed = 0;
            t.max_ns = p.max_wait_ns;
            for (uint32_t s = 0; s < kTmaStages; ++s)
                asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&tma_bar[w.wi][s])) : "memory");
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
    }
    const uint32_t nwarps = gridDim.x * kWarps;
    JobRing *jr = p.jobs;
    // Active-job bitmap: 32 words right after the ring (see job_ring_bytes()).
    uint32_t *bits = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(p.jobs) +
                                                  sizeof(JobRing));
    const uint64_t t_launch = gtime();
    const bool leader = w.wi == 0;
    if (threadIdx.x < 32) s_bits[threadIdx.x] = ld_vol32(&bits[threadIdx.x]);
    w.mr_epoch = &s_epoch;
    w.epoch = 0;
    if (threadIdx.x == 0) {
        s_slots = ld_vol32(&p.stats->qp_slots);
        s_epoch = ld_vol32(&p.stats->mr_epoch);
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
        const uint32_t orank = owner_rank(w.wi);
        const bool owner = blockIdx.x + gridDim.x * orank < slots;
        bool in_flight = false;  // an owned QP waits for WRs to finish: come back to it soon
        for (uint32_t q = blockIdx.x + gridDim.x * orank; q < slots; q += gridDim.x * kWarps) {
            work += service_qp(w, &p.qps[q], wqe_buf[w.wi], cqe_buf[w.wi], jr, bits, nwarps);
            if (w.abort) {
                s_exit = 1;
                flush_counters(w);
                return;
            }
            in_flight |= w.vq == &p.qps[q] && w.vhead != w.vissue;
        }
        if (!leader) {
            // A warp whose QPs have WRs in flight takes one chunk per round, so it notices their
            // completion (and retires them) within one chunk's time rather than eight.
            const int max_chunks = in_flight ? 1 : 8;
            for (int k = 0; k < max_chunks; ++k) {
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
                    s_epoch = ld_vol32(&p.stats->mr_epoch);
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

constexpr size_t kTmaSmemBytes = kTmaBuilt ? size_t(kWarps - 1) * kTmaStages * kTmaPiece : 0;

int launch_executor(const ExecParams &p, int ctas, cudaStream_t stream) {
    // The dynamic shared memory (TMA staging) is above the 48 KiB default: opt in (cheap, and
    // per device, so it is set on every launch).
    if (kTmaSmemBytes > 0)
        if (cudaError_t e = cudaFuncSetAttribute(executor_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 int(kTmaSmemBytes));
            e != cudaSuccess)
            return int(e);
    executor_kernel<<<ctas, kThreads, kTmaSmemBytes, stream>>>(p);
    return int(cudaGetLastError());
}

int executor_kernels(const KernelRef **out) {
    static const KernelRef refs[] = {
        {"executor_kernel", reinterpret_cast<const void *>(&executor_kernel), kThreads},
        {"grid_copy_kernel", reinterpret_cast<const void *>(&grid_copy_kernel), kThreads},
        {"copy_test_kernel", reinterpret_cast<const void *>(&copy_test_kernel), 32},
    };
    *out = refs;
    return int(sizeof(refs) / sizeof(refs[0]));
}

int launch_copy_test(void *dst, const void *src, uint64_t n, cudaStream_t stream) {
    copy_test_kernel<<<1, 32, 0, stream>>>(static_cast<uint8_t *>(dst),
                                           static_cast<const uint8_t *>(src), n);
    return int(cudaGetLastError());
}

}  // namespace ugdr::gpu
