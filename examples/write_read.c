/* A complete ugdr client in C11: one RDMA WRITE, one RDMA READ and one FETCH_ADD between two
 * connected QPs, over memory of the device named on the command line ("ugdr_cpu0" for the daemon's
 * host-memory engine, which needs no GPU).  Build and run:
 *
 *   cc -std=c11 -Iinclude examples/write_read.c -Lugdr_b200/_lib -lugdr \
 *      -Wl,-rpath,ugdr_b200/_lib -o write_read
 *   ugdr_b200/_lib/ugdr_daemon --socket /tmp/ugdr.sock --gpus 0 &
 *   UGDR_DAEMON_SOCKET=/tmp/ugdr.sock ./write_read ugdr_cpu0
 *
 * GPU memory works the same way: register cudaMalloc ranges with ugdr_reg_mr on a GPU device.
 */
#include "ugdr/api.hpp"

#include <errno.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

static int wait_one(ugdr_cq *cq, uint64_t wr_id) {
    ugdr_wc wc;
    for (long spin = 0; spin < 100000000L; ++spin) {
        const int n = ugdr_poll_cq(cq, 1, &wc);
        if (n < 0) return -n;
        if (n == 1) return (wc.status == UGDR_WC_SUCCESS && wc.wr_id == wr_id) ? 0 : EIO;
    }
    return ETIMEDOUT;
}

static int post1(ugdr_qp *qp, ugdr_send_wr *wr) {
    ugdr_send_wr *bad = NULL;
    return ugdr_post_send(qp, wr, &bad);
}

int main(int argc, char **argv) {
    const char *want = argc > 1 ? argv[1] : "ugdr_cpu0";
    int n = 0;
    ugdr_device **list = ugdr_get_device_list(&n);
    if (list == NULL) {
        fprintf(stderr, "no daemon: %s\n", strerror(errno));
        return 1;
    }
    ugdr_device *dev = NULL;
    for (int i = 0; i < n; ++i) {
        ugdr_x_device_info info;
        if (ugdr_x_query_device(list[i], &info) == 0 && strcmp(info.name, want) == 0) dev = list[i];
    }
    if (dev == NULL) {
        fprintf(stderr, "no device %s\n", want);
        return 1;
    }
    ugdr_context *ctx = ugdr_open_device(dev);
    ugdr_pd *pd = ugdr_alloc_pd(ctx);
    ugdr_cq *cq = ugdr_create_cq(ctx, 64, NULL, NULL, 0);
    const size_t len = 1 << 16;
    uint8_t *buf = (uint8_t *)ugdr_x_alloc_host(len); /* host memory the daemon can map */
    const int acc = UGDR_ACCESS_LOCAL_WRITE | UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_READ |
                    UGDR_ACCESS_REMOTE_ATOMIC;
    ugdr_mr *mr = buf ? ugdr_reg_mr(pd, buf, len, acc) : NULL;
    ugdr_qp_init_attr ia = {cq, cq, 16, 16, 1, 1, UGDR_QPT_RC, 0};
    ugdr_qp *a = ugdr_create_qp(pd, &ia), *b = ugdr_create_qp(pd, &ia);
    if (!ctx || !pd || !cq || !mr || !a || !b) {
        fprintf(stderr, "setup failed: %s\n", strerror(errno));
        return 1;
    }
    /* RESET -> INIT with remote access, then connect each side to the other (INIT -> RTS). */
    ugdr_qp_attr at;
    memset(&at, 0, sizeof(at));
    at.qp_state = UGDR_QPS_INIT;
    at.qp_access_flags = UGDR_ACCESS_REMOTE_WRITE | UGDR_ACCESS_REMOTE_READ | UGDR_ACCESS_REMOTE_ATOMIC;
    ugdr_modify_qp(a, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS);
    ugdr_modify_qp(b, &at, UGDR_QP_STATE | UGDR_QP_ACCESS_FLAGS);
    ugdr_qp_conn_info ca, cb;
    ugdr_query_qp_conn_info(a, &ca);
    ugdr_query_qp_conn_info(b, &cb);
    ugdr_qp_attr ct;
    memset(&ct, 0, sizeof(ct));
    ct.timeout = 14;
    ct.retry_cnt = 7;
    ct.rnr_retry = 7;
    ct.min_rnr_timer = 1;
    const int cm = UGDR_QP_TIMEOUT | UGDR_QP_RETRY_CNT | UGDR_QP_RNR_RETRY | UGDR_QP_MIN_RNR_TIMER;
    if (ugdr_connect_qp(a, &cb, &ct, cm) || ugdr_connect_qp(b, &ca, &ct, cm)) {
        fprintf(stderr, "connect failed\n");
        return 1;
    }

    for (int i = 0; i < 256; ++i) buf[i] = (uint8_t)i;
    ugdr_sge sg = {(uint64_t)(uintptr_t)buf, 256, mr->lkey};
    ugdr_send_wr wr;
    memset(&wr, 0, sizeof(wr));
    wr.sg_list = &sg;
    wr.num_sge = 1;
    wr.send_flags = UGDR_SEND_SIGNALED;

    /* WRITE bytes [0, 256) to [4096, 4352). */
    wr.wr_id = 1;
    wr.opcode = UGDR_WR_RDMA_WRITE;
    wr.wr.rdma.remote_addr = (uint64_t)(uintptr_t)(buf + 4096);
    wr.wr.rdma.rkey = mr->rkey;
    if (post1(a, &wr) || wait_one(cq, 1) || memcmp(buf, buf + 4096, 256) != 0) return 2;

    /* READ them back into [8192, 8448). */
    sg.addr = (uint64_t)(uintptr_t)(buf + 8192);
    wr.wr_id = 2;
    wr.opcode = UGDR_WR_RDMA_READ;
    if (post1(a, &wr) || wait_one(cq, 2) || memcmp(buf, buf + 8192, 256) != 0) return 3;

    /* FETCH_ADD 5 to the counter at 12288; the old value lands at 12296. */
    uint64_t *counter = (uint64_t *)(buf + 12288), *old = (uint64_t *)(buf + 12296);
    *counter = 37;
    sg.addr = (uint64_t)(uintptr_t)old;
    sg.length = 8;
    wr.wr_id = 3;
    wr.opcode = UGDR_WR_ATOMIC_FETCH_AND_ADD;
    memset(&wr.wr, 0, sizeof(wr.wr));
    wr.wr.atomic.remote_addr = (uint64_t)(uintptr_t)counter;
    wr.wr.atomic.compare_add = 5;
    wr.wr.atomic.rkey = mr->rkey;
    if (post1(a, &wr) || wait_one(cq, 3) || *old != 37 || *counter != 42) return 4;

    ugdr_destroy_qp(a);
    ugdr_destroy_qp(b);
    ugdr_dereg_mr(mr);
    ugdr_x_free_host(buf);
    ugdr_destroy_cq(cq);
    ugdr_dealloc_pd(pd);
    ugdr_close_device(ctx);
    ugdr_free_device_list(list);
    printf("write, read and fetch-add ok on %s\n", want);
    return 0;
}
