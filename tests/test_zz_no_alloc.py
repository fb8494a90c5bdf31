"""The allocation-free GDN prefill entry point
(wkvm_chunk_gated_delta_rule_static) against the workspace-taking one.

It exists for hosts that cannot allocate device memory while serving (device
memory owned by their own pool, or a cgo / JNI embedding without an
allocator): its scratch is a fixed array inside the library. The test calls
it through the C ABI twice in a row, with different inputs and one input
long enough to need several windows of the array, and checks each result
against wkvm_chunk_gated_delta_rule. This file is collected last."""

import ctypes

import pytest
import torch

from conftest import REL_TOL, assert_out_close, rel_err
from wkvm_b200 import _lib, ops, synth

pytestmark = pytest.mark.gpu

GDN = ("q", "k", "v", "g", "beta")


def _static_call(d, scale):
    q = d["q"]
    B, T, H, K = q.shape
    HV, V = d["v"].shape[2], d["v"].shape[3]
    o = torch.empty_like(d["v"])
    ht = torch.empty(B, HV, K, V, dtype=torch.float32, device=q.device)
    status = ops.status_word(q.device)
    P = ctypes.c_void_p
    rc = _lib.load().wkvm_chunk_gated_delta_rule_static(
        *(P(d[n].data_ptr()) for n in GDN), P(o.data_ptr()), P(d["h0"].data_ptr()),
        P(ht.data_ptr()), None, B, T, H, HV, K, V, ctypes.c_float(scale), 1,
        1, P(status.data_ptr()), P(torch.cuda.current_stream(q.device).cuda_stream))
    assert rc == 0, _lib.WkvmError("wkvm_chunk_gated_delta_rule_static", rc)
    return o, ht


@pytest.mark.parametrize("calls", [[(2, 300, 2, 4, 5), (1, 64, 2, 2, 6)],
                                   [(16, 2048, 4, 8, 7), (3, 129, 1, 1, 8)]])
def test_static_scratch_matches_workspace_path(cuda, calls):
    # (B, T, H, HV, seed): 16 x 8 heads x 32 chunks does not fit the array in
    # one window, so that call runs in windows
    for B, T, H, HV, seed in calls:
        x = synth.gdn_inputs(B, T, H, 128, HV=HV, seed=seed)
        d = {n: t.to(cuda) for n, t in x.items()}
        scale = 128 ** -0.5
        o, ht = _static_call(d, scale)
        ro, rh = ops.chunk_gated_delta_rule(*(d[n] for n in GDN), scale=scale,
                                            initial_state=d["h0"], output_final_state=True,
                                            use_qk_l2norm_in_kernel=True)
        ops.check_device_status(cuda)
        assert_out_close(o, ro.float())
        assert rel_err(ht, rh) < REL_TOL


def test_static_scratch_rejects_oversized_batch(cuda):
    # one chunk record and one carried state per (sequence, value head) no
    # longer fit the 64 MiB array
    lib = _lib.load()
    nseq, T = 1000, 128
    one_window = lib.wkvm_gdn_chunk_workspace_bytes(nseq, 64, 1, 128, 128) + nseq * 128 * 128 * 4
    assert one_window > 2 * (64 << 20)
    # real buffers of the stated shape (about 260 MB), so that a regression in
    # the size check gives a wrong answer, never an access outside memory
    x = synth.gdn_inputs(nseq, T, 1, 128, seed=9)
    d = {n: t.to(cuda) for n, t in x.items()}
    o = torch.empty_like(d["v"])
    ht = torch.empty_like(d["h0"])
    P = ctypes.c_void_p
    rc = lib.wkvm_chunk_gated_delta_rule_static(
        *(P(d[n].data_ptr()) for n in GDN), P(o.data_ptr()), P(d["h0"].data_ptr()),
        P(ht.data_ptr()), None, nseq, T, 1, 1, 128, 128, ctypes.c_float(1.0), 0, 1,
        None, P(torch.cuda.current_stream(cuda).cuda_stream))
    torch.cuda.synchronize()
    assert rc == -10
    assert lib.wkvm_strerror(rc) == b"request larger than the static scratch array"
