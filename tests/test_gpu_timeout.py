"""The bounded-wait failure path of the streamed kernels, driven without any fault.

Every mbarrier wait in the streamed kernels gives up after a bound, records LOOM_SELECT_ETIMEOUT in
the workspace and winds its CTA down (the producer stops issuing, the copies already issued are
drained). The test hook loom_select_test_wait_fault lowers that bound to 50 us and makes the first
CTA's producer leave one stage unissued, so its consumers' waits run out: nothing faults, traps or
waits without a bound. The call must report the timeout, and after loom_select_workspace_init the
next call on the same workspace must be exact again (against the oracle).
"""
import numpy as np
import pytest
import torch

import synth

pytestmark = pytest.mark.gpu
NT = 8
LIMIT_NS = 50_000


def _arm(sel, ws, withhold):
    lib = sel.lib()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.loom_select_test_wait_fault(ws.buf.data_ptr(), LIMIT_NS, withhold, stream) == sel.OK


def _reset(sel, ws):
    lib = sel.lib()
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.loom_select_workspace_init(ws.buf.data_ptr(), ws.buf.numel(), stream) == sel.OK


def test_sampler_wait_runs_out_then_next_call_is_exact(sel, dev, oracle):
    x, hist, u = synth.sample_chain(64, seed=21, device="cuda")   # split rows: records and tickets too
    ws = sel.Workspace(dev)
    sel.sample_rows(x, u, 0.7, 1.1, 40, 0.9, history=hist, workspace=ws)   # sizes the workspace
    torch.cuda.synchronize()
    assert ws.read_status() == sel.OK
    _arm(sel, ws, 1)
    sel.sample_rows(x, u, 0.7, 1.1, 40, 0.9, history=hist, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == sel.ETIMEOUT
    _reset(sel, ws)
    ids, prob = sel.sample_rows(x, u, 0.7, 1.1, 40, 0.9, history=hist, workspace=ws)
    torch.cuda.synchronize()
    want = oracle.sample_rows(x.cpu().numpy(), u.cpu().numpy(), 0.7, 1.1, 40, 0.9, hist.cpu().numpy(), nthreads=NT)
    np.testing.assert_array_equal(ids.cpu().numpy(), want["ids"])
    np.testing.assert_allclose(prob.cpu().numpy(), want["prob"], rtol=1e-5)
    assert ws.read_status() == sel.OK


def test_argmax_wait_runs_out_then_next_call_is_exact(sel, dev, oracle):
    x, _, _ = synth.sample_chain(128, seed=22, device="cuda")     # 19.4 M elements: the streamed kernel
    ws = sel.Workspace(dev)
    out = torch.empty(128, dtype=torch.int32, device=dev)
    sel.argmax_rows_into(x, out, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == sel.OK
    _arm(sel, ws, 2)
    sel.argmax_rows_into(x, out, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == sel.ETIMEOUT
    _reset(sel, ws)
    sel.argmax_rows_into(x, out, workspace=ws)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.argmax_rows(x.cpu().numpy(), nthreads=NT))
    assert ws.read_status() == sel.OK


def test_hook_rejects_bad_arguments(sel, dev):
    lib = sel.lib()
    ws = sel.Workspace(dev)
    buf = ws.get(4096)
    assert lib.loom_select_test_wait_fault(None, LIMIT_NS, 0, None) == sel.EWORKSPACE
    assert lib.loom_select_test_wait_fault(buf.data_ptr(), 0, 0, None) == sel.EINVAL
    assert lib.loom_select_test_wait_fault(buf.data_ptr(), LIMIT_NS, -2, None) == sel.EINVAL


def test_lm_head_wait_runs_out_then_next_call_is_exact(sel, dev):
    # the fused LM-head kernel: CTA 0's producer leaves its 4th K slice unissued, the MMA warp's wait
    # runs out, every role winds down (copies and MMAs issued are drained, TMEM is freed)
    g = torch.Generator(device="cuda").manual_seed(31)
    h = torch.randn(64, 512, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(20000, 512, generator=g, device="cuda") / 22.6).to(torch.bfloat16)
    ws = sel.Workspace(dev)
    ids0, _, _ = sel.lm_head_argmax(h, w, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == sel.OK
    _arm(sel, ws, 3)
    sel.lm_head_argmax(h, w, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == sel.ETIMEOUT
    _reset(sel, ws)
    ids, logit, lse = sel.lm_head_argmax(h, w, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == sel.OK
    assert torch.equal(ids, ids0)
    ref = h.float() @ w.float().t()
    assert bool((ref.gather(1, ids.long()[:, None])[:, 0] >= ref.max(dim=1).values - 2e-3).all())
    assert torch.allclose(lse, torch.logsumexp(ref, dim=1), atol=2e-3, rtol=0)
