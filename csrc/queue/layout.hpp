// Byte layouts shared by the client, the daemon and the device executors.
//
// These layouts are a wire format: a v1 client of the reference (src/queue/shared_ring.hpp:26-51,
// src/queue/descriptors.hpp:11-81) must be able to exchange rings with this daemon, so every
// offset below is fixed and static_assert-checked.  The header is plain C++ with no library
// types so the same definitions compile into CUDA device code.
//
// Ring header (192 B): metadata line, producer cursor line (`tail`), consumer cursor line
// (`head`); slots start at byte 192.  Cursors grow monotonically; slot = cursor % capacity.
//
// Extensions in reserved space (v1 readers never look at these):
//  * metadata.reserved[0] of a send ring is the QP error word: the daemon / executor stores
//    UGDR_QPS_ERR there when the QP enters ERR so the client posting path can see it.
//  * Atomic send WQEs (opcodes 5 and 6) carry exactly one SGE; `swap` is split across
//    `immediate_data` (low 32 bits) and `reserved` (high 32 bits), and `compare_add` is the
//    8-byte word that follows the SGE (offset 56), so an atomic WQE still fits a 64-byte slot.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace ugdr::queue {

constexpr uint32_t kRingMagic = 0x55475251u;  // "UGRQ"
constexpr uint16_t kRingVersion = 1;
constexpr uint32_t kLine = 64;
constexpr uint32_t kRingHeaderBytes = 3 * kLine;
constexpr uint32_t kSlotAlign = 64;

enum RingKind : uint16_t { kSendRing = 1, kRecvRing = 2, kCompletionRing = 3 };

struct alignas(64) RingMeta {
    uint32_t magic;
    uint16_t version;
    uint16_t kind;
    uint32_t header_bytes;
    uint32_t reserved0;
    uint64_t mapping_bytes;
    uint32_t capacity;
    uint32_t slot_stride;
    uint64_t reserved[4];
};

struct alignas(64) RingCursor {
    uint64_t value;
    uint64_t pad[7];
};

struct alignas(64) RingHeader {
    RingMeta meta;
    RingCursor tail;  // producer cursor
    RingCursor head;  // consumer cursor
};

struct Sge {
    uint64_t address;
    uint32_t length;
    uint32_t lkey;
};

struct SendWqe {
    uint64_t wr_id;
    uint64_t remote_address;
    uint32_t rkey;
    uint32_t opcode;
    uint32_t send_flags;
    uint32_t immediate_data;
    uint32_t sge_count;
    uint32_t reserved;
};

struct RecvWqe {
    uint64_t wr_id;
    uint32_t sge_count;
    uint32_t reserved;
};

struct Cqe {
    uint64_t wr_id;
    uint32_t status;
    uint32_t opcode;
    uint32_t byte_length;
    uint32_t immediate_data;
    uint32_t qp_num;
    uint32_t flags;
};

static_assert(sizeof(RingMeta) == 64, "ring metadata is one line");
static_assert(sizeof(RingCursor) == 64, "cursor is one line");
static_assert(sizeof(RingHeader) == kRingHeaderBytes, "ring header is 192 bytes");
static_assert(offsetof(RingHeader, tail) == 64 && offsetof(RingHeader, head) == 128, "cursors");
static_assert(offsetof(RingMeta, mapping_bytes) == 16 && offsetof(RingMeta, capacity) == 24,
              "metadata offsets");
static_assert(sizeof(Sge) == 16 && sizeof(SendWqe) == 40 && sizeof(RecvWqe) == 16 &&
                  sizeof(Cqe) == 32,
              "descriptor sizes");
static_assert(offsetof(SendWqe, rkey) == 16 && offsetof(SendWqe, sge_count) == 32,
              "send WQE offsets");

// Offset of the first SGE inside a slot, per ring kind.
constexpr uint32_t kSendSgeOffset = sizeof(SendWqe);
constexpr uint32_t kRecvSgeOffset = sizeof(RecvWqe);
// Atomic operand position (see the file comment).
constexpr uint32_t kAtomicCompareOffset = kSendSgeOffset + sizeof(Sge);

// Slot stride = header + max_sge SGEs rounded up to 64 B; 0 on overflow.
constexpr uint32_t slot_stride_for(uint32_t header, uint32_t max_sge) {
    const uint64_t raw = uint64_t(header) + uint64_t(max_sge) * sizeof(Sge);
    const uint64_t rounded = (raw + kSlotAlign - 1) / kSlotAlign * kSlotAlign;
    return rounded > 0xffffffffull ? 0u : uint32_t(rounded);
}
constexpr uint32_t send_stride(uint32_t max_sge) { return slot_stride_for(40, max_sge); }
constexpr uint32_t recv_stride(uint32_t max_sge) { return slot_stride_for(16, max_sge); }
constexpr uint32_t completion_stride() { return kSlotAlign; }

constexpr uint32_t kQpErrorWordIndex = 0;  // metadata.reserved[0] of the send ring

}  // namespace ugdr::queue
