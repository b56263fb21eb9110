"""ctypes view of libugdr.so: the public C ABI of include/ugdr/api.hpp.

The structures mirror the header field for field (the same layouts the reference exposes in
include/ugdr/api.hpp:13-204, plus the appended READ / atomic members).  The library is built
in-tree by `make` into ugdr_b200/_lib/; importing this module without it raises, so no caller
silently falls back to a Python path.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_DIR = Path(os.environ.get("UGDR_LIB_DIR") or Path(__file__).resolve().parent / "_lib")
LIB_PATH = LIB_DIR / "libugdr.so"
# UGDR_DAEMON_BIN selects another daemon build (e.g. the sanitizer one) for the launcher.
DAEMON_PATH = Path(os.environ.get("UGDR_DAEMON_BIN") or LIB_DIR / "ugdr_daemon")

# ---- enums (numeric values are libibverbs') -------------------------------------------------
QPT_RC = 2
QPS_RESET, QPS_INIT, QPS_RTR, QPS_RTS, QPS_SQD, QPS_SQE, QPS_ERR, QPS_UNKNOWN = range(8)
QP_STATE = 1 << 0
QP_CUR_STATE = 1 << 1
QP_ACCESS_FLAGS = 1 << 3
QP_TIMEOUT = 1 << 9
QP_RETRY_CNT = 1 << 10
QP_RNR_RETRY = 1 << 11
QP_MIN_RNR_TIMER = 1 << 15
CONNECT_MASK = QP_TIMEOUT | QP_RETRY_CNT | QP_RNR_RETRY | QP_MIN_RNR_TIMER

WR_RDMA_WRITE = 0
WR_RDMA_WRITE_WITH_IMM = 1
WR_RDMA_READ = 4
WR_ATOMIC_CMP_AND_SWP = 5
WR_ATOMIC_FETCH_AND_ADD = 6
WR_X_RDMA_WRITE_SUM_BF16 = 24  # extension: WRITE of the elementwise bf16 sum of the SGEs
SEND_SIGNALED = 1 << 1

WC_SUCCESS = 0
WC_LOC_LEN_ERR = 1
WC_LOC_QP_OP_ERR = 2
WC_LOC_PROT_ERR = 4
WC_WR_FLUSH_ERR = 5
WC_LOC_ACCESS_ERR = 8
WC_REM_INV_REQ_ERR = 9
WC_REM_ACCESS_ERR = 10
WC_REM_OP_ERR = 11
WC_RETRY_EXC_ERR = 12
WC_RNR_RETRY_EXC_ERR = 13
WC_GENERAL_ERR = 21

WC_RDMA_WRITE = 1
WC_RDMA_READ = 2
WC_COMP_SWAP = 3
WC_FETCH_ADD = 4
WC_RECV_RDMA_WITH_IMM = 129
WC_WITH_IMM = 1 << 1

ACCESS_LOCAL_WRITE = 1 << 0
ACCESS_REMOTE_WRITE = 1 << 1
ACCESS_REMOTE_READ = 1 << 2
ACCESS_REMOTE_ATOMIC = 1 << 3


class Mr(C.Structure):
    _fields_ = [
        ("context", C.c_void_p),
        ("pd", C.c_void_p),
        ("addr", C.c_void_p),
        ("length", C.c_size_t),
        ("handle", C.c_uint32),
        ("lkey", C.c_uint32),
        ("rkey", C.c_uint32),
    ]


class Sge(C.Structure):
    _fields_ = [("addr", C.c_uint64), ("length", C.c_uint32), ("lkey", C.c_uint32)]


class _Rdma(C.Structure):
    _fields_ = [("remote_addr", C.c_uint64), ("rkey", C.c_uint32)]


class _Atomic(C.Structure):
    _fields_ = [
        ("remote_addr", C.c_uint64),
        ("compare_add", C.c_uint64),
        ("swap", C.c_uint64),
        ("rkey", C.c_uint32),
    ]


class _WrUnion(C.Union):
    _fields_ = [("rdma", _Rdma), ("atomic", _Atomic)]


class SendWr(C.Structure):
    pass


SendWr._fields_ = [
    ("wr_id", C.c_uint64),
    ("next", C.POINTER(SendWr)),
    ("sg_list", C.POINTER(Sge)),
    ("num_sge", C.c_int),
    ("opcode", C.c_int),
    ("send_flags", C.c_uint),
    ("imm_data", C.c_uint32),
    ("wr", _WrUnion),
]


class RecvWr(C.Structure):
    pass


RecvWr._fields_ = [
    ("wr_id", C.c_uint64),
    ("next", C.POINTER(RecvWr)),
    ("sg_list", C.POINTER(Sge)),
    ("num_sge", C.c_int),
]


class Wc(C.Structure):
    _fields_ = [
        ("wr_id", C.c_uint64),
        ("status", C.c_int),
        ("opcode", C.c_int),
        ("vendor_err", C.c_uint32),
        ("byte_len", C.c_uint32),
        ("imm_data", C.c_uint32),
        ("qp_num", C.c_uint32),
        ("src_qp", C.c_uint32),
        ("wc_flags", C.c_uint),
        ("pkey_index", C.c_uint16),
        ("slid", C.c_uint16),
        ("sl", C.c_uint8),
        ("dlid_path_bits", C.c_uint8),
    ]


class QpInitAttr(C.Structure):
    _fields_ = [
        ("send_cq", C.c_void_p),
        ("recv_cq", C.c_void_p),
        ("max_send_wr", C.c_uint32),
        ("max_recv_wr", C.c_uint32),
        ("max_send_sge", C.c_uint32),
        ("max_recv_sge", C.c_uint32),
        ("qp_type", C.c_int),
        ("sq_sig_all", C.c_int),
    ]


class QpAttr(C.Structure):
    _fields_ = [
        ("qp_state", C.c_int),
        ("cur_qp_state", C.c_int),
        ("qp_access_flags", C.c_int),
        ("timeout", C.c_uint8),
        ("retry_cnt", C.c_uint8),
        ("rnr_retry", C.c_uint8),
        ("min_rnr_timer", C.c_uint8),
    ]


class QpConnInfo(C.Structure):
    _fields_ = [("qp_num", C.c_uint32)]


class DeviceInfo(C.Structure):
    _fields_ = [
        ("name", C.c_char * 32),
        ("kind", C.c_int),
        ("gpu_ordinal", C.c_int),
        ("identity", C.c_uint64),
    ]


class DaemonStats(C.Structure):
    _fields_ = [(f, C.c_uint64) for f in ("devices", "contexts", "pds", "mrs", "cqs", "qps")]


class QpStats(C.Structure):
    _fields_ = [
        ("send_posted", C.c_uint64),
        ("send_retired", C.c_uint64),
        ("recv_posted", C.c_uint64),
        ("recv_consumed", C.c_uint64),
        ("bytes", C.c_uint64),
        ("error_completions", C.c_uint64),
        ("rnr_waits", C.c_uint64),
        ("state", C.c_uint32),
        ("reserved", C.c_uint32),
    ]


class EngineStats(C.Structure):
    _fields_ = [
        ("wrs_completed", C.c_uint64),
        ("bytes_moved", C.c_uint64),
        ("error_completions", C.c_uint64),
        ("launches", C.c_uint64),
        ("wait_timeouts", C.c_uint64),
        ("first_start_ns", C.c_uint64),
        ("last_end_ns", C.c_uint64),
        ("chunks_run", C.c_uint64),
        ("claim_misses", C.c_uint64),
        ("jobs_published", C.c_uint64),
        ("inline_runs", C.c_uint64),
        ("busy_ns", C.c_uint64),
        ("fast_batches", C.c_uint64),
        ("fast_fetch_ns", C.c_uint64),
        ("fast_exec_ns", C.c_uint64),
        ("fast_reserve_ns", C.c_uint64),
        ("fast_publish_ns", C.c_uint64),
        ("slow_wrs", C.c_uint64),
        ("slow_issue_ns", C.c_uint64),
        ("job_slot_misses", C.c_uint64),
        ("publish_waits", C.c_uint64),
        ("publish_wait_ns", C.c_uint64),
        ("mr_detach_live", C.c_uint64),
        ("mr_detach_quiesced", C.c_uint64),
        ("order_waits", C.c_uint64),
        ("overlap_issues", C.c_uint64),
    ]


_lib = None


def lib() -> C.CDLL:
    """Load libugdr.so (once).  Raises if the in-tree build is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build the native library first (make -j, or "
            "`python -c 'import __graft_entry__ as g; g.build()'`)"
        )
    L = C.CDLL(str(LIB_PATH), mode=C.RTLD_GLOBAL, use_errno=True)
    vp, i, u32, u64, sz = C.c_void_p, C.c_int, C.c_uint32, C.c_uint64, C.c_size_t
    sig = {
        "ugdr_get_device_list": (C.POINTER(vp), [C.POINTER(i)]),
        "ugdr_free_device_list": (None, [C.POINTER(vp)]),
        "ugdr_open_device": (vp, [vp]),
        "ugdr_close_device": (i, [vp]),
        "ugdr_alloc_pd": (vp, [vp]),
        "ugdr_dealloc_pd": (i, [vp]),
        "ugdr_reg_mr": (C.POINTER(Mr), [vp, vp, sz, i]),
        "ugdr_dereg_mr": (i, [C.POINTER(Mr)]),
        "ugdr_create_cq": (vp, [vp, i, vp, vp, i]),
        "ugdr_destroy_cq": (i, [vp]),
        "ugdr_poll_cq": (i, [vp, i, C.POINTER(Wc)]),
        "ugdr_create_qp": (vp, [vp, C.POINTER(QpInitAttr)]),
        "ugdr_destroy_qp": (i, [vp]),
        "ugdr_modify_qp": (i, [vp, C.POINTER(QpAttr), i]),
        "ugdr_query_qp": (i, [vp, C.POINTER(QpAttr), i, C.POINTER(QpInitAttr)]),
        "ugdr_query_qp_conn_info": (i, [vp, C.POINTER(QpConnInfo)]),
        "ugdr_connect_qp": (i, [vp, C.POINTER(QpConnInfo), C.POINTER(QpAttr), i]),
        "ugdr_post_send": (i, [vp, C.POINTER(SendWr), C.POINTER(C.POINTER(SendWr))]),
        "ugdr_post_recv": (i, [vp, C.POINTER(RecvWr), C.POINTER(C.POINTER(RecvWr))]),
        "ugdr_x_query_device": (i, [vp, C.POINTER(DeviceInfo)]),
        "ugdr_x_reg_mr_multicast": (C.POINTER(Mr), [vp, vp, sz, i, i]),
        "ugdr_x_alloc_host": (vp, [sz]),
        "ugdr_x_free_host": (i, [vp]),
        "ugdr_x_query_engine_stats": (i, [vp, C.POINTER(EngineStats), i]),
        "ugdr_x_query_qp_stats": (i, [vp, C.POINTER(QpStats)]),
        "ugdr_x_query_daemon_stats": (i, [C.POINTER(DaemonStats)]),
        "ugdr_x_poll_cq_wait": (i, [vp, i, i, C.POINTER(Wc), C.c_uint64]),
        "ugdr_x_engine_trace": (i, [vp, C.c_uint32]),
        "ugdr_x_engine_trace_dump": (i, [vp, C.c_char_p, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
        "ugdr_x_engine_hold": (i, [vp, i]),
        "ugdr_x_timed_drain": (i, [C.POINTER(vp), i, C.POINTER(u64), u32, C.POINTER(C.c_float)]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def errno() -> int:
    return C.get_errno()


def errname(code: int) -> str:
    return os.strerror(code) if code > 0 else "ok"
