#include "api/posting.hpp"

#include <cerrno>
#include <cstring>

namespace ugdr::api {
namespace {

bool is_atomic(uint32_t op) {
    return op == UGDR_WR_ATOMIC_CMP_AND_SWP || op == UGDR_WR_ATOMIC_FETCH_AND_ADD;
}

// Opcodes a send WQE may carry, as a bit mask over the opcode value.
constexpr uint32_t kSendOpMask = (1u << UGDR_WR_RDMA_WRITE) | (1u << UGDR_WR_RDMA_WRITE_WITH_IMM) |
                                 (1u << UGDR_WR_RDMA_READ) | (1u << UGDR_WR_ATOMIC_CMP_AND_SWP) |
                                 (1u << UGDR_WR_ATOMIC_FETCH_AND_ADD) | (1u << UGDR_X_WR_RDMA_WRITE_SUM_BF16);

inline bool send_ok(const ugdr_send_wr &wr, uint32_t max_sge) {
    const uint32_t op = uint32_t(wr.opcode);
    if (op >= 32 || ((kSendOpMask >> op) & 1u) == 0) return false;
    if ((wr.send_flags & ~unsigned(UGDR_SEND_SIGNALED)) != 0) return false;
    if (wr.num_sge < 0 || uint32_t(wr.num_sge) > max_sge) return false;
    if (wr.num_sge > 0 && wr.sg_list == nullptr) return false;
    if (is_atomic(wr.opcode) && wr.num_sge != 1) return false;
    return true;
}

bool recv_ok(const ugdr_recv_wr &wr, uint32_t max_sge) {
    if (wr.num_sge < 0 || uint32_t(wr.num_sge) > max_sge) return false;
    if (wr.num_sge > 0 && wr.sg_list == nullptr) return false;
    return true;
}

template <typename Wr, typename Ok, typename Enc>
int post_chain(queue::Ring &ring, Wr *wr, Wr **bad_wr, Ok ok, Enc enc) {
    if (wr == nullptr || bad_wr == nullptr) {
        if (bad_wr) *bad_wr = wr;
        return EINVAL;
    }
    // One pass: take the slots known to be free, validate and encode WRs into them in order,
    // publish the encoded prefix once.  The consumer cursor (a line the consumer writes) is
    // re-read only when those slots run out.
    queue::SlotRun run = ring.reserve_free(false);
    uint32_t room = run.count();
    const uint32_t stride = ring.geometry().stride;
    uint8_t *slot = run.first;
    uint32_t left_in_span = run.first_count;
    uint32_t n = 0;
    int err = 0;
    Wr *w = wr;
    for (; w != nullptr; w = w->next) {
        if (!ok(*w)) {
            err = EINVAL;
            break;
        }
        if (n == room) {
            ring.publish(n);
            run = ring.reserve_free(true);
            room = run.count();
            slot = run.first;
            left_in_span = run.first_count;
            n = 0;
            if (room == 0) {
                err = ENOMEM;
                break;
            }
        }
        if (left_in_span == 0) {  // wrapped into the second span
            slot = run.second;
            left_in_span = run.second_count;
        }
        enc(slot, *w);
        slot += stride;
        --left_in_span;
        ++n;
    }
    ring.publish(n);
    if (err != 0) {
        *bad_wr = w;
        return err;
    }
    return 0;
}

}  // namespace

void encode_send(uint8_t *slot, const ugdr_send_wr &wr) {
    // Slots are 64-byte aligned, so the header is written in place, field by field.
    auto *h = reinterpret_cast<queue::SendWqe *>(slot);
    h->wr_id = wr.wr_id;
    h->opcode = uint32_t(wr.opcode);
    h->send_flags = wr.send_flags;
    h->sge_count = uint32_t(wr.num_sge);
    if (is_atomic(wr.opcode)) {
        h->remote_address = wr.wr.atomic.remote_addr;
        h->rkey = wr.wr.atomic.rkey;
        h->immediate_data = uint32_t(wr.wr.atomic.swap);
        h->reserved = uint32_t(wr.wr.atomic.swap >> 32);
        std::memcpy(slot + queue::kAtomicCompareOffset, &wr.wr.atomic.compare_add, 8);
    } else {
        h->remote_address = wr.wr.rdma.remote_addr;
        h->rkey = wr.wr.rdma.rkey;
        h->immediate_data = wr.opcode == UGDR_WR_RDMA_WRITE_WITH_IMM ? wr.imm_data : 0;
        h->reserved = 0;
    }
    auto *sg = reinterpret_cast<queue::Sge *>(slot + queue::kSendSgeOffset);
    for (int i = 0; i < wr.num_sge; ++i) sg[i] = queue::Sge{wr.sg_list[i].addr, wr.sg_list[i].length, wr.sg_list[i].lkey};
}

void encode_recv(uint8_t *slot, const ugdr_recv_wr &wr) {
    queue::RecvWqe h{wr.wr_id, uint32_t(wr.num_sge), 0};
    std::memcpy(slot, &h, sizeof(h));
    for (int i = 0; i < wr.num_sge; ++i) {
        queue::Sge s{wr.sg_list[i].addr, wr.sg_list[i].length, wr.sg_list[i].lkey};
        std::memcpy(slot + queue::kRecvSgeOffset + i * sizeof(queue::Sge), &s, sizeof(s));
    }
}

int post_send_chain(queue::Ring &sq, uint32_t max_sge, ugdr_send_wr *wr, ugdr_send_wr **bad_wr) {
    return post_chain(sq, wr, bad_wr, [max_sge](const ugdr_send_wr &w) { return send_ok(w, max_sge); },
                      encode_send);
}

int post_recv_chain(queue::Ring &rq, uint32_t max_sge, ugdr_recv_wr *wr, ugdr_recv_wr **bad_wr) {
    return post_chain(rq, wr, bad_wr, [max_sge](const ugdr_recv_wr &w) { return recv_ok(w, max_sge); },
                      encode_recv);
}

void cqe_to_wc(const queue::Cqe &c, ugdr_wc *wc) {
    std::memset(wc, 0, sizeof(*wc));
    wc->wr_id = c.wr_id;
    wc->status = ugdr_wc_status(c.status);
    wc->opcode = ugdr_wc_opcode(c.opcode);
    wc->byte_len = c.byte_length;
    wc->imm_data = c.immediate_data;
    wc->qp_num = c.qp_num;
    wc->wc_flags = c.flags;
}

}  // namespace ugdr::api
