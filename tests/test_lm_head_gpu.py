"""The lm_head + argmax kernel (w4_lm_head_argmax) at full vocabulary against a float64 oracle.

The decode step ends with the final RMSNorm, the tied bf16 lm_head and a
greedy argmax (scripts/decode_loop.py:117-118 ran them as the HF forward's
last ops and torch.argmax). Here the kernel is called through the C ABI on
the Qwen2.5-1.5B shape (vocab 151936, hidden 1536) and on two others, and
compared with oracle/decode_oracle.py's float64 logits: every logit within
bf16 rounding, the token equal to the oracle's argmax wherever the top two
logits are apart by more than that, ties resolved to the lowest row (as
torch.argmax does), and the position advanced by one.
"""
import numpy as np
import pytest
import torch

from oracle.decode_oracle import lm_head_logits_f64

pytestmark = pytest.mark.gpu

from roofline_decoding_b200 import _lib  # noqa: E402

DEV = "cuda"
EPS = 1e-6


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _run(lib, h, norm_w, embed, vocab, hidden):
    ws = torch.zeros((int(lib.w4_lm_head_workspace_bytes()),), dtype=torch.uint8, device=DEV)
    logits = torch.empty((vocab,), dtype=torch.bfloat16, device=DEV)
    token = torch.zeros(1, dtype=torch.long, device=DEV)
    pos = torch.full((1,), 41, dtype=torch.long, device=DEV)
    _lib.check(lib.w4_lm_head_argmax(h.data_ptr(), norm_w.data_ptr(), EPS, embed.data_ptr(),
                                     vocab, hidden, logits.data_ptr(), token.data_ptr(),
                                     pos.data_ptr(), ws.data_ptr(), ws.numel(), 0,
                                     torch.cuda.current_stream().cuda_stream),
               "w4_lm_head_argmax")
    torch.cuda.synchronize()
    assert int(pos.item()) == 42
    assert not ws.any(), "the workspace is left zeroed for the next step"
    return logits.float().cpu().double().numpy(), int(token.item())


@pytest.mark.parametrize("vocab,hidden", [(151936, 1536), (1001, 256), (50000, 2048)])
def test_lm_head_argmax_matches_float64_oracle(vocab, hidden):
    lib = _lib.load()
    g = torch.Generator(device="cpu").manual_seed(vocab + hidden)
    h = torch.randn((hidden,), generator=g).to(torch.bfloat16)
    norm_w = (1.0 + 0.05 * torch.randn((hidden,), generator=g)).to(torch.bfloat16)
    embed = (0.02 * torch.randn((vocab, hidden), generator=g)).to(torch.bfloat16)
    want = lm_head_logits_f64(_bits(h), _bits(norm_w), _bits(embed), EPS)
    got, tok = _run(lib, h.to(DEV), norm_w.to(DEV), embed.to(DEV), vocab, hidden)
    scale = np.abs(want).max()
    err = np.abs(got - want)
    # a bf16 store (2^-9 relative) plus fp32 accumulation over `hidden` terms
    assert (err <= 2.0 ** -8 * np.abs(want) + 1e-5 * scale).all(), float(err.max())
    assert tok == int(np.argmax(got)), "token = first maximum of the kernel's own logits"
    top2 = np.sort(want)[-2:]
    if top2[1] - top2[0] > 2.0 ** -7 * abs(top2[1]):
        assert tok == int(np.argmax(want))


def test_lm_head_argmax_ties_pick_the_lowest_row():
    lib = _lib.load()
    vocab, hidden = 151936, 1536
    g = torch.Generator(device="cpu").manual_seed(5)
    h = torch.randn((hidden,), generator=g).to(torch.bfloat16)
    norm_w = torch.ones((hidden,)).to(torch.bfloat16)
    embed = (0.01 * torch.randn((vocab, hidden), generator=g)).to(torch.bfloat16)
    winner = embed[0].clone()
    winner.copy_((0.2 * torch.sign(h.float())).to(torch.bfloat16))  # a clear maximum
    rows = [150000, 7777, 70001, 151935]  # the same row at several places, in other CTAs
    for r in rows:
        embed[r] = winner
    _, tok = _run(lib, h.to(DEV), norm_w.to(DEV), embed.to(DEV), vocab, hidden)
    assert tok == min(rows)
