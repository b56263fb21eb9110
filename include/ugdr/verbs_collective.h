/* Collectives built on the ugdr verbs: every byte moves as an RDMA WRITE work request that the
 * daemon's persistent executors run, the reduction is the UGDR_X_WR_RDMA_WRITE_SUM_BF16 opcode
 * (the sum is done by the executor while it writes the result), and ranks signal each other with
 * WRITE_WITH_IMM receive completions.  No counterpart in the reference (it has no collectives);
 * they use only its public object model: registered MRs, connected RC QPs, one CQ.
 *
 * A group is wired by the caller (see ugdr_b200.parallel.verbs_collectives for a torch
 * version): each rank opens a context on its GPU, creates one CQ, registers its data buffer and
 * a staging buffer, creates per peer one QP that writes to that peer (`to`) and one that the
 * peer writes through (`from`, whose receive queue takes the peer's immediates), plus a
 * connected loopback pair on its own GPU (`self_to`), and exchanges addresses and rkeys.
 *
 * Sizes: the send queues of `to` and `self_to` hold at least 2 x pieces WRs, the receive queue
 * of each `from` QP at least 2 x pieces WRs, max_send_sge of `self_to` is at least n, and the CQ
 * has room for 2 x pieces x (n - 1) + pieces + n entries. */
#pragma once

#include "ugdr/api.hpp"

#ifdef __cplusplus
#define UGDR_VC_NOEXCEPT noexcept
extern "C" {
#else
#define UGDR_VC_NOEXCEPT
#endif

#define UGDR_X_VGROUP_MAX_RANKS 8

typedef struct ugdr_x_vgroup_peer {
    ugdr_qp *to;         /* connected to this peer's `from` QP for our rank */
    ugdr_qp *from;       /* connected to this peer's `to` QP for our rank */
    uint64_t buf_addr;   /* the peer's data buffer */
    uint32_t buf_rkey;
    uint32_t stage_rkey;
    uint64_t stage_addr; /* the peer's staging buffer */
} ugdr_x_vgroup_peer;

typedef struct ugdr_x_vgroup {
    int rank;
    int n;
    ugdr_cq *cq;          /* send and receive CQ of every QP of the group */
    ugdr_qp *self_to;     /* loopback QP on this rank's GPU (connected to a local peer QP) */
    uint64_t buf_addr;    /* this rank's data buffer (registered as buf_lkey / buf_rkey) */
    uint32_t buf_lkey;
    uint32_t buf_rkey;
    uint64_t stage_addr;  /* n x shard-size bytes (registered as stage_lkey) */
    uint32_t stage_lkey;
    uint32_t pad;
    uint64_t stage_bytes;
    uint32_t epoch;       /* calls made so far (tags the immediates); start at 0 */
    uint32_t pad2;
    ugdr_x_vgroup_peer peer[UGDR_X_VGROUP_MAX_RANKS]; /* index = peer rank; own entry unused */
} ugdr_x_vgroup;

/* Staging bytes an allreduce of `count` bf16 elements over n ranks needs. */
uint64_t ugdr_x_verbs_allreduce_stage_bytes(uint64_t count, int n) UGDR_VC_NOEXCEPT;

/* In-place sum of `count` bf16 elements at buf_addr over the group (fp32 accumulation), as a
 * reduce-scatter and an all-gather of WRs, pipelined in `pieces` pieces per shard:
 *   1. rank r WRITE_WITH_IMMs piece m of shard q into rank q's staging slot r;
 *   2. once a piece of its shard arrived from every peer, rank r posts one WRITE_SUM_BF16 on
 *      its loopback QP whose n SGEs are the ranks' pieces in rank order (its own in place, the
 *      others staged), written in place over its own piece, so each element is the fp32 sum
 *      x_0 + ... + x_{n-1} rounded to bf16 once;
 *   3. when that sum completes, rank r WRITE_WITH_IMMs the piece to every peer's buffer.
 * Every rank calls it with the same count and pieces.  Blocks until this rank's part is done
 * (its buffer holds the sum and its WRs retired).  Each call first posts its own receives; a
 * peer that runs ahead waits in RNR (the `to` QPs need rnr_retry 7) until they are posted, so
 * no call's data lands in a buffer still in use by the previous one.  Returns 0, EINVAL,
 * ETIMEDOUT (nothing for timeout_ns), EIO (an error completion) or an errno of the verbs calls. */
int ugdr_x_verbs_allreduce_bf16(ugdr_x_vgroup *g, uint64_t count, int pieces,
                                uint64_t timeout_ns) UGDR_VC_NOEXCEPT;

/* The same sum through NVLink SHARP: `mc_addr` is this process's multicast view of an NVLS
 * object holding the data (every rank's unicast copy at the same offsets), registered on this
 * rank's PD with ugdr_x_reg_mr_multicast (mc_lkey / mc_rkey).  After a ready exchange (zero-length
 * WRITE_WITH_IMMs), each rank posts ONE UGDR_X_WR_RDMA_WRITE_SUM_BF16 on its loopback QP whose
 * source and destination are its shard in the multicast view: the executor's multimem loads have
 * the NVSwitch sum the shard over every GPU (fp32 accumulation) and its multimem stores write the
 * sum to every GPU; a second exchange tells every rank that every shard is done.  Per GPU about
 * (1 + 1/n) of the buffer crosses each link direction.  count a multiple of 8, mc_addr 16-byte
 * aligned.  Returns 0, EINVAL, ETIMEDOUT, EIO or a verbs errno. */
int ugdr_x_verbs_allreduce_bf16_mc(ugdr_x_vgroup *g, uint64_t mc_addr, uint32_t mc_lkey, uint32_t mc_rkey,
                                   uint64_t count, uint64_t timeout_ns) UGDR_VC_NOEXCEPT;

/* MoE all-to-all on the verbs.  Experts split evenly over the ranks (rank q owns experts
 * [q * nexp / n, (q + 1) * nexp / n)).  The permutes are the SGE lists of the WRs: dispatch
 * WRITEs gather each expert group's token rows (one SGE per row) into one contiguous range of
 * the owner's receive area; combine READs each group back in one piece.  The group's `to` QPs and `self_to` need
 * max_send_sge >= 32 and send queues of at least ugdr_x_verbs_moe_wrs(...) WRs; `from` QPs need
 * 2 receives per call.  Counts travel as WRITE_WITH_IMM into every rank's count table (a host
 * buffer), which also orders calls: a rank's next dispatch writes nothing before every rank has
 * finished its combine. */
typedef struct ugdr_x_vmoe {
    int tokens;
    int topk;
    int nexp;
    uint32_t row_bytes;
    uint64_t x_addr;        /* [tokens][row_bytes] rows to send (registered: x_lkey) */
    uint32_t x_lkey;
    uint32_t recv_lkey;
    uint64_t recv_addr;     /* receive area: recv_rows rows, grouped by expert then source rank */
    uint32_t recv_rkey;
    uint32_t back_lkey;
    uint64_t recv_rows;
    uint64_t back_addr;     /* [tokens * topk][row_bytes]: rows read back, grouped by expert */
    int32_t *table;         /* host [n][nexp] counts (registered: table_lkey / table_rkey) */
    uint32_t table_lkey;
    uint32_t table_rkey;
    uint64_t peer_recv_addr[UGDR_X_VGROUP_MAX_RANKS];
    uint32_t peer_recv_rkey[UGDR_X_VGROUP_MAX_RANKS];
    uint64_t peer_table_addr[UGDR_X_VGROUP_MAX_RANKS];
    uint32_t peer_table_rkey[UGDR_X_VGROUP_MAX_RANKS];
    /* Filled by dispatch for combine: first receive row of (expert e, source rank r) at the
     * owner, and how many rows this rank received. */
    uint64_t *base;         /* host [nexp][n] */
    uint64_t received;
} ugdr_x_vmoe;

/* Largest number of data WRs one dispatch or combine posts on one QP for `rows_per_rank`
 * (token, k) rows (an upper bound for sizing send queues). */
uint32_t ugdr_x_verbs_moe_wrs(uint64_t rows_per_rank, int nexp, int n) UGDR_VC_NOEXCEPT;

/* Send every (token, k) row to its expert's owner.  `ids` and `pos` (host, tokens x topk int32)
 * are each row's expert and its position inside this rank's rows of that expert (row order, as
 * ugdr_x_moe_route gives them); `counts` (host, nexp int32) this rank's rows per expert.  Blocks
 * until this rank's rows have landed and every peer's rows for this rank's experts have too.
 * Returns 0, ENOSPC (receive area too small), EINVAL, ETIMEDOUT, EIO or a verbs errno. */
int ugdr_x_verbs_moe_dispatch(ugdr_x_vgroup *g, ugdr_x_vmoe *m, const int32_t *ids, const int32_t *pos,
                              const int32_t *counts, uint64_t timeout_ns) UGDR_VC_NOEXCEPT;

/* The same from rows already grouped by expert: `back` holds this rank's tokens * topk rows,
 * expert e's from row sum_{e' < e} counts[e'] on (as ugdr_x_moe_pack_grouped writes them), and
 * each (owner, expert) group leaves as ONE contiguous WRITE, which the executors split into
 * chunks over all their warps.  Same result, completions and errors as the gathering form. */
int ugdr_x_verbs_moe_dispatch_packed(ugdr_x_vgroup *g, ugdr_x_vmoe *m, const int32_t *counts,
                                     uint64_t timeout_ns) UGDR_VC_NOEXCEPT;

/* Read every row this rank dispatched (after the owners' experts worked on them in place) back
 * into `back`, grouped by expert in the order dispatch sent them: expert e's rows start at row
 * sum_{e' < e} counts[e'], in position order.  Each (owner, expert) group is ONE contiguous READ;
 * ugdr_x_moe_weighted_sum_grouped then unpermutes and weights them in one pass.  Blocks until
 * all reads completed. */
int ugdr_x_verbs_moe_combine(ugdr_x_vgroup *g, ugdr_x_vmoe *m, uint64_t timeout_ns) UGDR_VC_NOEXCEPT;

#ifdef __cplusplus
}
#endif
#undef UGDR_VC_NOEXCEPT
