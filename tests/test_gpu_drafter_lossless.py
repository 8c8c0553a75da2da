"""The reference's end-to-end lossless test with the real draft stack
(``tests/test_generate_lossless.py:72-86``): ``dsm.drafter.DSparkDrafter`` (stage 0's embedding
and main projection, the whole DSpark block -- attention and FFN hyper-connection halves
around the sparse attention and the MoE -- and the Markov draft head, all on ``libdsm``)
drafts against the order-1 Markov base in the restated greedy loop of ``generate.py:39-88``.

1. Lockstep with the oracle drafter: both drafters get the same calls (the loop follows the
   oracle's drafts) and their drafts must agree block by block, position by position, up to the
   first position where the oracle's biased logits hold a near tie; the biased logits agree
   within 2e-2 of their scale until there (fp32 activations, weights held as f16 in the packed
   tiles: 2^-11 relative each, through two hyper-connection halves and the head).
2. The GPU drafter driving the loop alone: the emitted 20 tokens equal plain greedy decoding of
   the base, as the reference asserts.
"""

from __future__ import annotations

import pytest
import torch

import oracle
from drafter_case import N_NEW, MAX_SEQ_LEN, base_and_prompt, drafter_weights, full_args, generate, plain_greedy
from dsm import _lib
from dsm.drafter import DSparkDrafter

pytestmark = pytest.mark.gpu
DEV = "cuda"
ATOL = 2e-2


def _gpu_drafter(t: dict, a: dict) -> DSparkDrafter:
    d = DSparkDrafter(a, max_seq_len=MAX_SEQ_LEN).to(DEV)
    for name, v in t.items():
        *path, leaf = name.split(".")
        obj = d
        for p in path:
            obj = getattr(obj, p)
        if leaf in obj._buffers:
            setattr(obj, leaf, v.to(DEV))
        else:
            setattr(obj, leaf, torch.nn.Parameter(v.to(DEV), requires_grad=False))
    return d


class _Lockstep:
    """Drives the oracle drafter (whose drafts the loop follows) and the GPU drafter with the
    same calls, keeping both outputs of every drafted block."""

    def __init__(self, ref, gpu):
        self.ref, self.gpu, self.blocks = ref, gpu, []

    def forward_spec(self, input_ids, main_hidden, start_pos=0):
        out_ref = self.ref.forward_spec(input_ids.cpu(), main_hidden.cpu(), start_pos)
        out_gpu = self.gpu.forward_spec(input_ids.to(DEV), main_hidden.to(DEV), start_pos)
        if start_pos:
            torch.cuda.synchronize()
            self.blocks.append((out_ref, tuple(o.cpu() for o in out_gpu)))
        return out_ref

    def advance(self, main_hidden, position):
        self.ref.advance(main_hidden.cpu(), position)
        self.gpu.advance(main_hidden.to(DEV), position)


def test_drafter_drafts_match_oracle_and_stream_is_lossless():
    a = full_args()
    t = drafter_weights(a)
    transition, embed, prompt = base_and_prompt()
    lock = _Lockstep(oracle.OracleDrafter(t, a, MAX_SEQ_LEN), _gpu_drafter(t, a))
    tokens = generate(lock, transition, embed, prompt, N_NEW)
    assert tokens == plain_greedy(transition, prompt[-1], N_NEW)
    assert _lib.device_error() == 0
    compared = 0
    for b, ((ids_r, lg_r, conf_r), (ids_g, lg_g, conf_g)) in enumerate(lock.blocks):
        assert ids_g.shape == ids_r.shape and lg_g.shape == lg_r.shape
        assert int(ids_g[0, 0]) == int(ids_r[0, 0])  # the anchor
        for i in range(lg_r.shape[1]):
            scale = max(1.0, float(lg_r[0, i].abs().max()))
            assert float((lg_g[0, i] - lg_r[0, i]).abs().max()) <= ATOL * scale, (b, i)
            compared += 1
            if int(ids_g[0, i + 1]) != int(ids_r[0, i + 1]):
                top2 = torch.topk(lg_r[0, i], 2).values
                assert float(top2[0] - top2[1]) <= 2 * ATOL * scale, (b, i, "drafts differ without a near tie")
                break
    assert compared >= len(lock.blocks)  # at least every block's first draft position


def test_gpu_drafter_drives_the_loop_losslessly():
    a = full_args()
    transition, embed, prompt = base_and_prompt()
    gpu = _gpu_drafter(drafter_weights(a), a)
    tokens = generate(gpu, transition, embed, prompt, N_NEW, device=DEV)
    assert len(tokens) == N_NEW
    assert tokens == plain_greedy(transition, prompt[-1], N_NEW)
    assert _lib.device_error() == 0
