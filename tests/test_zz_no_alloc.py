"""ksh_lm_head_argmax_noalloc: the lm_head + greedy argmax entry point that
keeps its scratch in a fixed device array instead of a caller workspace.

It is checked against ksh_lm_head_argmax (the workspace entry point) on the
same inputs, for two calls in a row, at the tolerance the other lm_head tests
use (logits within 1e-5 of the largest |logit|; tokens identical).  The file
name sorts last so it also runs after every other GPU test.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

TOO_LARGE = -6


def _workspace_call(lib, xc, m, H, nw, wc, V):
    logits = torch.empty((m, V), device="cuda")
    tok = torch.empty(m, dtype=torch.int64, device="cuda")
    ws = torch.zeros(int(lib.lib().ksh_lm_head_workspace_size(m, V)), dtype=torch.uint8,
                     device="cuda")
    lib.call("ksh_lm_head_argmax", xc.data_ptr(), m, H, nw, 1e-6, wc.data_ptr(), V,
             logits.data_ptr(), tok.data_ptr(), ws.data_ptr(), ws.numel(), lib.stream_ptr())
    torch.cuda.synchronize()
    return logits.cpu(), tok.cpu()


@pytest.mark.parametrize("m,V,H,norm", [(1, 151936, 896, True), (4, 151936, 896, False),
                                        (16, 32000, 2048, True), (3, 1000, 64, False)])
def test_noalloc_matches_workspace_entry_two_calls(m, V, H, norm):
    from kshipra_b200 import _lib
    gen = torch.Generator().manual_seed(m * 7 + V + H)
    w = torch.randn((V, H), generator=gen) * 0.02
    w[V // 3] = w[V - 5]                  # exact tie: the lower index must win
    x = torch.randn((m, H), generator=gen)
    x[0] = w[V - 5] * 50
    nwt = (1.0 + 0.1 * torch.randn(H, generator=gen)).cuda() if norm else None
    nw = nwt.data_ptr() if norm else None
    wc, xc = w.cuda(), x.cuda()
    ref_logits, ref_tok = _workspace_call(_lib, xc, m, H, nw, wc, V)
    scale = float(ref_logits.abs().max())
    for _ in range(2):
        logits = torch.full((m, V), float("nan"), device="cuda")
        tok = torch.full((m,), -1, dtype=torch.int64, device="cuda")
        _lib.call("ksh_lm_head_argmax_noalloc", xc.data_ptr(), m, H, nw, 1e-6, wc.data_ptr(), V,
                  logits.data_ptr(), tok.data_ptr(), _lib.stream_ptr())
        torch.cuda.synchronize()
        lg = logits.cpu()
        assert float((lg - ref_logits).abs().max()) <= 1e-5 * scale
        assert tok.cpu().tolist() == ref_tok.tolist()
        assert int(tok[0]) == V // 3
    # argmax-only call (no logits buffer) gives the same tokens
    tok = torch.full((m,), -1, dtype=torch.int64, device="cuda")
    _lib.call("ksh_lm_head_argmax_noalloc", xc.data_ptr(), m, H, nw, 1e-6, wc.data_ptr(), V, None,
              tok.data_ptr(), _lib.stream_ptr())
    torch.cuda.synchronize()
    assert tok.cpu().tolist() == ref_tok.tolist()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from kshipra_b200 import _lib
    h = _lib.lib()
    assert h.ksh_lm_head_argmax_noalloc_max_bytes() == 256 * 1024
    assert h.ksh_status_string(TOO_LARGE) != b"unknown status"
    x = torch.zeros((17, 64), device="cuda")
    w = torch.zeros((1000, 64), device="cuda")
    tok = torch.empty(17, dtype=torch.int64, device="cuda")
    # 17 rows: more than the fixed scratch is sized for; refused before any launch
    st = h.ksh_lm_head_argmax_noalloc(x.data_ptr(), 17, 64, None, 0.0, w.data_ptr(), 1000, None,
                                      tok.data_ptr(), _lib.stream_ptr())
    assert st == TOO_LARGE


def test_noalloc_scratch_covers_this_gpus_argmax_grid():
    """The largest argmax grid on this GPU (8 CTAs per SM) fits the array for 16 rows."""
    from kshipra_b200 import _lib
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert 256 + sms * 8 * 16 * 8 <= _lib.lib().ksh_lm_head_argmax_noalloc_max_bytes()
