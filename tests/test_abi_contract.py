"""ABI contract of the public headers (reference suite semantics: tests/unit/api_contract_c_test.c
compiles the header as C11; libibverbs_alignment_test.cpp pins values and layouts).

* include/ugdr/api.hpp, include/ugdr/collective.h and include/ugdr/route_noalloc.h compile as strict C11.
* Enum values are libibverbs' (ibv_wr_opcode, ibv_wc_status, ibv_wc_opcode, ibv_qp_state,
  ibv_access_flags, ibv_qp_attr_mask bits), written out here because <infiniband/verbs.h> is not
  installed on this machine.
* The ctypes structures of the Python binding have the C compiler's sizes and field offsets.
"""
from __future__ import annotations

import ctypes as C
import os
import shutil
import subprocess
import tempfile

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

IBV_VALUES = {
    "UGDR_QPT_RC": 2,
    "UGDR_QPS_RESET": 0, "UGDR_QPS_INIT": 1, "UGDR_QPS_RTR": 2, "UGDR_QPS_RTS": 3, "UGDR_QPS_SQD": 4,
    "UGDR_QPS_SQE": 5, "UGDR_QPS_ERR": 6,
    "UGDR_QP_STATE": 1 << 0, "UGDR_QP_CUR_STATE": 1 << 1, "UGDR_QP_ACCESS_FLAGS": 1 << 3,
    "UGDR_QP_TIMEOUT": 1 << 9, "UGDR_QP_RETRY_CNT": 1 << 10, "UGDR_QP_RNR_RETRY": 1 << 11,
    "UGDR_QP_MIN_RNR_TIMER": 1 << 15,
    "UGDR_WR_RDMA_WRITE": 0, "UGDR_WR_RDMA_WRITE_WITH_IMM": 1, "UGDR_WR_RDMA_READ": 4,
    "UGDR_WR_ATOMIC_CMP_AND_SWP": 5, "UGDR_WR_ATOMIC_FETCH_AND_ADD": 6,
    "UGDR_SEND_SIGNALED": 1 << 1,
    "UGDR_WC_SUCCESS": 0, "UGDR_WC_LOC_LEN_ERR": 1, "UGDR_WC_LOC_QP_OP_ERR": 2, "UGDR_WC_LOC_PROT_ERR": 4,
    "UGDR_WC_WR_FLUSH_ERR": 5, "UGDR_WC_LOC_ACCESS_ERR": 8, "UGDR_WC_REM_INV_REQ_ERR": 9,
    "UGDR_WC_REM_ACCESS_ERR": 10, "UGDR_WC_REM_OP_ERR": 11, "UGDR_WC_RETRY_EXC_ERR": 12,
    "UGDR_WC_RNR_RETRY_EXC_ERR": 13, "UGDR_WC_GENERAL_ERR": 21,
    "UGDR_WC_RDMA_WRITE": 1, "UGDR_WC_RDMA_READ": 2, "UGDR_WC_COMP_SWAP": 3, "UGDR_WC_FETCH_ADD": 4,
    "UGDR_WC_RECV_RDMA_WITH_IMM": 129, "UGDR_WC_WITH_IMM": 1 << 1,
    "UGDR_ACCESS_LOCAL_WRITE": 1, "UGDR_ACCESS_REMOTE_WRITE": 2, "UGDR_ACCESS_REMOTE_READ": 4,
    "UGDR_ACCESS_REMOTE_ATOMIC": 8,
}

STRUCTS = {
    "ugdr_mr": ["context", "pd", "addr", "length", "handle", "lkey", "rkey"],
    "ugdr_sge": ["addr", "length", "lkey"],
    "ugdr_send_wr": ["wr_id", "next", "sg_list", "num_sge", "opcode", "send_flags", "imm_data", "wr"],
    "ugdr_recv_wr": ["wr_id", "next", "sg_list", "num_sge"],
    "ugdr_wc": ["wr_id", "status", "opcode", "vendor_err", "byte_len", "imm_data", "qp_num", "src_qp", "wc_flags",
                "pkey_index", "slid", "sl", "dlid_path_bits"],
    "ugdr_qp_init_attr": ["send_cq", "recv_cq", "max_send_wr", "max_recv_wr", "max_send_sge", "max_recv_sge",
                          "qp_type", "sq_sig_all"],
    "ugdr_qp_attr": ["qp_state", "cur_qp_state", "qp_access_flags", "timeout", "retry_cnt", "rnr_retry",
                     "min_rnr_timer"],
}


def _compile_and_run(src: str) -> str:
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "abi.c")
        exe = os.path.join(d, "abi")
        with open(c, "w") as f:
            f.write(src)
        subprocess.run([cc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I",
                        os.path.join(REPO, "include"), c, "-o", exe], check=True, capture_output=True, text=True)
        return subprocess.run([exe], check=True, capture_output=True, text=True).stdout


def _probe() -> dict:
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "ugdr/api.hpp"', '#include "ugdr/collective.h"',
             '#include "ugdr/route_noalloc.h"', '#include "ugdr/verbs_collective.h"', "int main(void) {"]
    for name in IBV_VALUES:
        lines.append(f'    printf("{name} %lld\\n", (long long){name});')
    for st, fields in STRUCTS.items():
        lines.append(f'    printf("sizeof.{st} %zu\\n", sizeof(struct {st}));')
        for fd in fields:
            lines.append(f'    printf("offsetof.{st}.{fd} %zu\\n", offsetof(struct {st}, {fd}));')
    lines.append('    printf("sizeof.ugdr_x_peerset %zu\\n", sizeof(ugdr_x_peerset));')
    lines.append('    printf("sizeof.ugdr_x_nvls %zu\\n", sizeof(ugdr_x_nvls));')
    lines.append('    printf("sizeof.ugdr_x_qp_stats %zu\\n", sizeof(ugdr_x_qp_stats));')
    lines.append('    printf("sizeof.ugdr_x_engine_stats %zu\\n", sizeof(ugdr_x_engine_stats));')
    lines.append('    printf("sizeof.ugdr_x_kernel_attr %zu\\n", sizeof(ugdr_x_kernel_attr));')
    lines.append('    printf("sizeof.ugdr_x_daemon_stats %zu\\n", sizeof(ugdr_x_daemon_stats));')
    lines += ["    return 0;", "}"]
    out = {}
    for line in _compile_and_run("\n".join(lines) + "\n").splitlines():
        k, v = line.split()
        out[k] = int(v)
    return out


@pytest.fixture(scope="module")
def probe():
    return _probe()


def test_enum_values_are_libibverbs(probe):
    for name, want in IBV_VALUES.items():
        assert probe[name] == want, name


def test_python_binding_layouts_match_the_header(probe):
    from ugdr_b200 import _native as N
    from ugdr_b200.parallel.nvls import Nvls
    from ugdr_b200.parallel.peers import PeerSet

    py = {"ugdr_mr": N.Mr, "ugdr_sge": N.Sge, "ugdr_send_wr": N.SendWr, "ugdr_recv_wr": N.RecvWr, "ugdr_wc": N.Wc,
          "ugdr_qp_init_attr": N.QpInitAttr, "ugdr_qp_attr": N.QpAttr}
    for st, cls in py.items():
        assert C.sizeof(cls) == probe[f"sizeof.{st}"], st
        for fd in STRUCTS[st]:
            assert getattr(cls, fd).offset == probe[f"offsetof.{st}.{fd}"], f"{st}.{fd}"
    assert C.sizeof(PeerSet) == probe["sizeof.ugdr_x_peerset"]
    assert C.sizeof(Nvls) == probe["sizeof.ugdr_x_nvls"]
    assert C.sizeof(N.QpStats) == probe["sizeof.ugdr_x_qp_stats"]
    assert C.sizeof(N.EngineStats) == probe["sizeof.ugdr_x_engine_stats"]
    from ugdr_b200.ops import KernelAttr

    assert C.sizeof(KernelAttr) == probe["sizeof.ugdr_x_kernel_attr"]
    assert C.sizeof(N.DaemonStats) == probe["sizeof.ugdr_x_daemon_stats"]


def test_binding_constants_match_the_header(probe):
    from ugdr_b200 import _native as N

    pairs = {"WR_RDMA_WRITE": "UGDR_WR_RDMA_WRITE", "WR_RDMA_WRITE_WITH_IMM": "UGDR_WR_RDMA_WRITE_WITH_IMM",
             "WR_RDMA_READ": "UGDR_WR_RDMA_READ", "WR_ATOMIC_CMP_AND_SWP": "UGDR_WR_ATOMIC_CMP_AND_SWP",
             "WR_ATOMIC_FETCH_AND_ADD": "UGDR_WR_ATOMIC_FETCH_AND_ADD", "WC_WR_FLUSH_ERR": "UGDR_WC_WR_FLUSH_ERR",
             "WC_RNR_RETRY_EXC_ERR": "UGDR_WC_RNR_RETRY_EXC_ERR", "WC_RECV_RDMA_WITH_IMM": "UGDR_WC_RECV_RDMA_WITH_IMM",
             "ACCESS_REMOTE_ATOMIC": "UGDR_ACCESS_REMOTE_ATOMIC", "QPS_ERR": "UGDR_QPS_ERR"}
    for py, c in pairs.items():
        assert getattr(N, py) == probe[c], py


# The reference's public function set (its client-contract list: tools/client-contracts.json).
REFERENCE_SYMBOLS = [
    "ugdr_get_device_list", "ugdr_free_device_list", "ugdr_open_device", "ugdr_close_device", "ugdr_alloc_pd",
    "ugdr_dealloc_pd", "ugdr_reg_mr", "ugdr_dereg_mr", "ugdr_create_cq", "ugdr_destroy_cq", "ugdr_poll_cq",
    "ugdr_create_qp", "ugdr_destroy_qp", "ugdr_modify_qp", "ugdr_query_qp", "ugdr_query_qp_conn_info",
    "ugdr_connect_qp", "ugdr_post_send", "ugdr_post_recv",
]


def _declared_functions() -> set[str]:
    import re

    names = set()
    for h in ("api.hpp", "collective.h", "route_noalloc.h", "verbs_collective.h"):
        with open(os.path.join(REPO, "include", "ugdr", h)) as f:
            text = re.sub(r"/\*.*?\*/|//[^\n]*", "", f.read(), flags=re.S)
        names |= set(re.findall(r"\b(ugdr_[a-z0-9_]+)\s*\([^;{]*\)\s*(?:noexcept\s*)?(?:UGDR_[A-Z_]*NOEXCEPT\s*)?;", text))
    return names


def test_every_declared_function_is_exported_with_c_linkage():
    """Each `ugdr_*` function declared in the public headers is a defined, unmangled dynamic
    symbol of libugdr.so, and the reference's whole public set is among them."""
    nm = shutil.which("nm")
    if nm is None:
        pytest.skip("nm not available")
    from ugdr_b200 import _native as N

    out = subprocess.run([nm, "-D", "--defined-only", str(N.LIB_PATH)], check=True, capture_output=True,
                         text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.split()[-2:-1] == ["T"]}
    declared = _declared_functions()
    assert set(REFERENCE_SYMBOLS) <= declared
    missing = sorted(declared - exported)
    assert not missing, missing


def test_diagnostics_fail_cleanly_without_a_gpu():
    """Without a CUDA device the kernel reports and copy diagnostics return a CUDA error code
    (raised as RuntimeError by the binding) instead of crashing the process."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from ugdr_b200 import ops

    with pytest.raises(RuntimeError):
        ops.kernel_attributes()
