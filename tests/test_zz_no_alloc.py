"""qmv_chain_noalloc (grid-barrier counters in a fixed device array, nothing allocated by the call)
against qmv_chain with a caller-provided workspace, through the C ABI.

Collected last on purpose, so that a run stopping at the first failure has run every other test first.
The first call in a process looks the array's address up; that path is checked in a fresh subprocess,
and the in-process test checks the calls after every other GPU test has run.  The device's free memory
is the same before and after a call: nothing is allocated."""
import ctypes
import os
import subprocess
import sys
import textwrap

import pytest
import torch

from nemicli_terminal_b200 import _lib, chain, synth

pytestmark = pytest.mark.gpu

QMV_ERR_TOO_LARGE = 8
MAX_STAGES = 128


def _outputs(ch, h_mid):
    return [y.clone() for s in ch.stages for y in s.ys] + [h_mid.clone()]


def _poison(ch, h_mid):
    for s in ch.stages:
        for y in s.ys:
            y.fill_(float("nan"))
    h_mid.fill_(float("nan"))


def test_noalloc_chain_matches_workspace_chain_on_two_calls(cuda):
    mk = lambda fmt, n_out, n_in, s: (fmt, synth.blocks(fmt, n_out, n_in, seed=500 + s, device=cuda), n_out, n_in)  # noqa: E731
    layer = (mk("Q4_K", 4096, 4096, 1), mk("Q4_K", 1024, 4096, 2), mk("Q4_K", 1024, 4096, 3),
             mk("Q4_K", 4096, 4096, 4), mk("Q4_K", 14336, 4096, 5), mk("Q4_K", 14336, 4096, 6),
             mk("Q6_K", 4096, 14336, 7))
    h0 = synth.activations(1, 4096, seed=21, device=cuda)[0]
    wa = torch.rand(4096, device=cuda) + 0.5
    wf = torch.rand(4096, device=cuda) + 0.5
    st, h_mid, _ = chain.layer_stages(*layer, h_in=h0, resid_in=None, attn_norm=wa, ffn_norm=wf, first=True)
    ch = chain.Chain(st)
    _lib.device_status(clear=True, device=cuda)

    ch.run()                                         # the existing entry point, workspace from the caller
    torch.cuda.synchronize()
    ref = _outputs(ch, h_mid)

    L = _lib.load()
    stream = _lib.stream_ptr(cuda)
    got = []
    for _ in range(2):                               # the second call must find its counters cleared again
        _poison(ch, h_mid)
        rc = L.qmv_chain_noalloc(ch.arr, len(ch.stages), stream)
        assert rc == 0, L.qmv_status_string(rc).decode()
        torch.cuda.synchronize()
        got.append(_outputs(ch, h_mid))
    for outs in got:
        for a, b in zip(outs, ref):
            assert torch.equal(a, b)
    assert _lib.device_status(clear=True, device=cuda) == 0      # no barrier timed out
    free0 = torch.cuda.mem_get_info(cuda)[0]
    assert L.qmv_chain_noalloc(ch.arr, len(ch.stages), stream) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(cuda)[0] == free0                # the call allocated nothing


def test_noalloc_chain_refuses_more_stages_than_its_counters(cuda):
    L = _lib.load()
    big = (chain._Stage * (MAX_STAGES + 1))()
    rc = L.qmv_chain_noalloc(big, MAX_STAGES + 1, _lib.stream_ptr(cuda))
    assert rc == QMV_ERR_TOO_LARGE
    assert b"no-allocation" in L.qmv_status_string(rc)
    assert L.qmv_chain_noalloc(None, 4, _lib.stream_ptr(cuda)) != 0
    assert L.qmv_chain_noalloc(big, 0, _lib.stream_ptr(cuda)) != 0


_FRESH = textwrap.dedent("""
    import sys, torch
    sys.path.insert(0, {root!r})
    from nemicli_terminal_b200 import _lib, chain, synth
    dev = torch.device("cuda", 0)
    raw = synth.blocks("Q4_K", 4096, 4096, seed=3, device=dev)
    x = synth.activations(1, 4096, seed=4, device=dev)[0].contiguous()
    ch = chain.Chain([chain.Stage("Q4_K", [(raw, 4096)], 4096, chain.RAW, a=x, wait=False)])
    L = _lib.load()
    for _ in range(2):                    # the first call in this process looks the array up
        ch.stages[0].ys[0].fill_(float("nan"))
        rc = L.qmv_chain_noalloc(ch.arr, 1, _lib.stream_ptr(dev))
        assert rc == 0, L.qmv_status_string(rc)
        torch.cuda.synchronize()
        got = ch.stages[0].ys[0].clone()
        ch.run()
        torch.cuda.synchronize()
        assert torch.equal(got, ch.stages[0].ys[0])
    print("fresh ok")
""")


def test_noalloc_first_call_in_a_fresh_process(cuda):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _FRESH.format(root=root)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "fresh ok" in r.stdout, r.stderr[-3000:]
