#include "api/posting.hpp"

#include <cerrno>
#include <cstring>

namespace ugdr::api {
namespace {

bool is_atomic(uint32_t op) {
    return op == UGDR_WR_ATOMIC_CMP_AND_SWP || op == UGDR_WR_ATOMIC_FETCH_AND_ADD;
}

bool send_ok(const ugdr_send_wr &wr, uint32_t max_sge) {
    switch (wr.opcode) {
    case UGDR_WR_RDMA_WRITE:
    case UGDR_WR_RDMA_WRITE_WITH_IMM:
    case UGDR_WR_RDMA_READ:
    case UGDR_WR_ATOMIC_CMP_AND_SWP:
    case UGDR_WR_ATOMIC_FETCH_AND_ADD: break;
    default: return false;
    }
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
    // Count the chain up to the first invalid WR, then reserve once.
    uint32_t want = 0;
    Wr *stop = nullptr;
    int err = 0;
    for (Wr *w = wr; w != nullptr; w = w->next) {
        if (!ok(*w)) {
            stop = w;
            err = EINVAL;
            break;
        }
        ++want;
    }
    queue::SlotRun run = ring.reserve(want);
    const uint32_t got = run.count();
    Wr *w = wr;
    const uint32_t stride = ring.geometry().stride;
    for (uint32_t i = 0; i < got; ++i, w = w->next) {
        uint8_t *slot = i < run.first_count ? run.first + uint64_t(i) * stride
                                            : run.second + uint64_t(i - run.first_count) * stride;
        enc(slot, *w);
    }
    ring.publish(got);
    if (got < want) {
        *bad_wr = w;
        return ENOMEM;
    }
    if (err != 0) {
        *bad_wr = stop;
        return err;
    }
    return 0;
}

}  // namespace

void encode_send(uint8_t *slot, const ugdr_send_wr &wr) {
    queue::SendWqe h;
    h.wr_id = wr.wr_id;
    h.opcode = uint32_t(wr.opcode);
    h.send_flags = wr.send_flags;
    h.sge_count = uint32_t(wr.num_sge);
    if (is_atomic(wr.opcode)) {
        h.remote_address = wr.wr.atomic.remote_addr;
        h.rkey = wr.wr.atomic.rkey;
        h.immediate_data = uint32_t(wr.wr.atomic.swap);
        h.reserved = uint32_t(wr.wr.atomic.swap >> 32);
        std::memcpy(slot + queue::kAtomicCompareOffset, &wr.wr.atomic.compare_add, 8);
    } else {
        h.remote_address = wr.wr.rdma.remote_addr;
        h.rkey = wr.wr.rdma.rkey;
        h.immediate_data = wr.opcode == UGDR_WR_RDMA_WRITE_WITH_IMM ? wr.imm_data : 0;
        h.reserved = 0;
    }
    std::memcpy(slot, &h, sizeof(h));
    for (int i = 0; i < wr.num_sge; ++i) {
        queue::Sge s{wr.sg_list[i].addr, wr.sg_list[i].length, wr.sg_list[i].lkey};
        std::memcpy(slot + queue::kSendSgeOffset + i * sizeof(queue::Sge), &s, sizeof(s));
    }
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
