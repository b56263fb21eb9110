// Data-path semantics shared by the CPU engine and (re-derived in device code) the GPU
// executor: opcode mapping, access rules, RNR timer decoding.
//
// Parity: reference contract docs/contracts/wr-wc-semantics.md (execution-condition table,
// WRITE_WITH_IMM responder rules); the reference worker implements WRITE / WRITE_WITH_IMM only
// (src/worker/worker.cpp:245-509) and stalls on an empty RQ instead of RNR
// (src/worker/worker.cpp:298-302).  This build implements RNR with the standard timer encoding.
#pragma once

#include "ugdr/api.hpp"

#include <cstdint>

namespace ugdr::engine {

inline bool op_known(uint32_t op) {
    return op == UGDR_WR_RDMA_WRITE || op == UGDR_WR_RDMA_WRITE_WITH_IMM || op == UGDR_WR_RDMA_READ ||
           op == UGDR_WR_ATOMIC_CMP_AND_SWP || op == UGDR_WR_ATOMIC_FETCH_AND_ADD ||
           op == UGDR_X_WR_RDMA_WRITE_SUM_BF16;
}
inline bool op_sum(uint32_t op) { return op == UGDR_X_WR_RDMA_WRITE_SUM_BF16; }

// fp32 -> bf16, round to nearest even (quiet NaN kept).  Plain IEEE-754 arithmetic on the bit
// pattern: add half an ulp of the bf16 result (plus the tie-to-even bit) and truncate.
inline uint16_t bf16_rne(float f) {
    uint32_t u;
    __builtin_memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return uint16_t(u >> 16);
}
inline float bf16_to_f32(uint16_t h) {
    const uint32_t u = uint32_t(h) << 16;
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
}
inline bool op_atomic(uint32_t op) {
    return op == UGDR_WR_ATOMIC_CMP_AND_SWP || op == UGDR_WR_ATOMIC_FETCH_AND_ADD;
}
inline uint32_t wc_opcode(uint32_t op) {
    switch (op) {
    case UGDR_WR_RDMA_READ: return UGDR_WC_RDMA_READ;
    case UGDR_WR_ATOMIC_CMP_AND_SWP: return UGDR_WC_COMP_SWAP;
    case UGDR_WR_ATOMIC_FETCH_AND_ADD: return UGDR_WC_FETCH_ADD;
    default: return UGDR_WC_RDMA_WRITE;
    }
}
// Remote MR / responder-QP access bit an opcode needs.
inline uint32_t remote_access_for(uint32_t op) {
    if (op == UGDR_WR_RDMA_READ) return UGDR_ACCESS_REMOTE_READ;
    if (op_atomic(op)) return UGDR_ACCESS_REMOTE_ATOMIC;
    return UGDR_ACCESS_REMOTE_WRITE;
}
// Local SGEs are written by READ and atomics (the fetched value).
inline bool local_written(uint32_t op) { return op == UGDR_WR_RDMA_READ || op_atomic(op); }

// Minimum RNR NAK timer, IB encoding 0..31, in nanoseconds (0 means 655.36 ms).
inline uint64_t rnr_timer_ns(uint8_t code) {
    static const uint32_t ten_us_units[32] = {
        65536, 1, 2, 3, 4, 6, 8, 12, 16, 24, 32, 48, 64, 96, 128, 192,
        256, 384, 512, 768, 1024, 1536, 2048, 3072, 4096, 6144, 8192, 12288, 16384, 24576, 32768, 49152};
    return uint64_t(ten_us_units[code & 31]) * 10000ull;  // (units of 10 us) -> ns
}
constexpr uint8_t kInfiniteRnrRetry = 7;

}  // namespace ugdr::engine
