// WR posting fast path: validate a linked WR chain and copy it into the QP's shared ring.
//
// Semantics follow the reference contract (docs/contracts/wr-wc-semantics.md "Posting and
// bad_wr"; implementation src/api/wr_posting.cpp:17-121): WRs are accepted in list order, the
// first invalid WR returns EINVAL and the first WR that finds the ring full returns ENOMEM, in
// both cases with *bad_wr naming it and the accepted prefix published.  One release store
// publishes the whole accepted prefix.  No allocation, syscall or lock beyond the caller's.
#pragma once

#include "queue/ring.hpp"
#include "ugdr/api.hpp"

#include <cstdint>

namespace ugdr::api {

int post_send_chain(queue::Ring &sq, uint32_t max_sge, ugdr_send_wr *wr, ugdr_send_wr **bad_wr);
int post_recv_chain(queue::Ring &rq, uint32_t max_sge, ugdr_recv_wr *wr, ugdr_recv_wr **bad_wr);

// Encode one send WR into a slot (no validation).  Exposed for tests and benchmarks.
void encode_send(uint8_t *slot, const ugdr_send_wr &wr);
void encode_recv(uint8_t *slot, const ugdr_recv_wr &wr);

// Translate a CQE into the public work completion.
void cqe_to_wc(const queue::Cqe &cqe, ugdr_wc *wc);

}  // namespace ugdr::api
