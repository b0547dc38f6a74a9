"""The allocation-free lm_head + argmax entry point (w4_lm_head_argmax_static).

It serves hosts that cannot give the library device memory: a C or C++
decode loop inside a process whose device memory belongs to another runtime,
or a plugin that may not allocate once it is serving. Its argmax state sits in
a fixed array inside the library instead of a caller workspace. This test
calls it through the C ABI twice in a row and checks each call against the
workspace entry point (w4_lm_head_argmax) on the same inputs: same logits
(within the bf16 tolerance the other tests use), same token, and the position
advanced by one per call. The file is named to be collected last; it runs the
same alone in a fresh process.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

from roofline_decoding_b200 import _lib  # noqa: E402

DEV = "cuda"
VOCAB, HIDDEN = 32003, 1536


def _inputs(seed, gain):
    g = torch.Generator(device="cpu").manual_seed(seed)
    h = torch.randn((1, HIDDEN), generator=g).to(torch.bfloat16).to(DEV)
    norm_w = (gain * (1.0 + 0.05 * torch.randn((HIDDEN,), generator=g))).to(torch.bfloat16)
    return h, norm_w.to(DEV)


def _call_workspace(lib, h, norm_w, embed, token, pos, ws, logits):
    st = lib.w4_lm_head_argmax(h.data_ptr(), norm_w.data_ptr(), 1e-6, embed.data_ptr(), VOCAB,
                               HIDDEN, logits.data_ptr(), token.data_ptr(), pos.data_ptr(),
                               ws.data_ptr(), ws.numel(), 0,
                               torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "w4_lm_head_argmax")


def _call_static(lib, h, norm_w, embed, token, pos, logits):
    st = lib.w4_lm_head_argmax_static(h.data_ptr(), norm_w.data_ptr(), 1e-6, embed.data_ptr(),
                                      VOCAB, HIDDEN, logits.data_ptr(), token.data_ptr(),
                                      pos.data_ptr(), 0, torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "w4_lm_head_argmax_static")


def test_static_scratch_matches_workspace_entry_point_twice():
    lib = _lib.load()
    g = torch.Generator(device="cpu").manual_seed(11)
    embed = (0.02 * torch.randn((VOCAB, HIDDEN), generator=g)).to(torch.bfloat16).to(DEV)
    ws = torch.zeros((int(lib.w4_lm_head_workspace_bytes()),), dtype=torch.uint8, device=DEV)
    tok_a = torch.zeros(1, dtype=torch.long, device=DEV)
    pos_a = torch.zeros(1, dtype=torch.long, device=DEV)
    tok_b = torch.zeros(1, dtype=torch.long, device=DEV)
    pos_b = torch.zeros(1, dtype=torch.long, device=DEV)
    best = []
    # the second call's logits are half as large: a state left over from the
    # first call would win its argmax and show up as a wrong token
    for call, (seed, gain) in enumerate(((1, 1.0), (2, 0.5))):
        h, norm_w = _inputs(seed, gain)
        logits_a = torch.empty((1, VOCAB), dtype=torch.bfloat16, device=DEV)
        logits_b = torch.empty((1, VOCAB), dtype=torch.bfloat16, device=DEV)
        _call_workspace(lib, h, norm_w, embed, tok_a, pos_a, ws, logits_a)
        _call_static(lib, h, norm_w, embed, tok_b, pos_b, logits_b)
        torch.cuda.synchronize()
        torch.testing.assert_close(logits_b.float(), logits_a.float(), rtol=2 ** -8, atol=1e-3)
        assert int(tok_b.item()) == int(tok_a.item()), f"call {call}"
        assert int(tok_b.item()) == int(torch.argmax(logits_b.float()).item())
        assert int(pos_b.item()) == call + 1 == int(pos_a.item())
        best.append(float(logits_b.float().max().item()))
    assert best[1] < best[0]
    assert _lib.device_error(torch.cuda.current_device()) == 0


def test_static_entry_point_rejects_out_of_range_sizes():
    lib = _lib.load()
    null = None
    st = lib.w4_lm_head_argmax_static(16, 16, 1e-6, 16, 0, HIDDEN, null, 16, 16, 0, null)
    assert st == _lib.W4_ERR_INVALID_ARG
    st = lib.w4_lm_head_argmax_static(16, 16, 1e-6, 16, VOCAB, 100, null, 16, 16, 0, null)
    assert st == _lib.W4_ERR_UNSUPPORTED
