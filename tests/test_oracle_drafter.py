"""The oracle drafter (``oracle.OracleDrafter``) in the reference's end-to-end lossless
scenario (``tests/test_generate_lossless.py:72-86``) on the CPU: the restated greedy loop with
the oracle's drafts emits exactly plain greedy decoding of the Markov base."""

from __future__ import annotations

import oracle
from drafter_case import N_NEW, MAX_SEQ_LEN, base_and_prompt, drafter_weights, full_args, generate, plain_greedy


def test_oracle_drafter_loop_is_lossless():
    a = full_args()
    transition, embed, prompt = base_and_prompt()
    drafter = oracle.OracleDrafter(drafter_weights(a), a, MAX_SEQ_LEN)
    blocks = []
    tokens = generate(drafter, transition, embed, prompt, N_NEW, on_block=lambda *b: blocks.append(b))
    assert len(tokens) == N_NEW
    assert tokens == plain_greedy(transition, prompt[-1], N_NEW)
    assert len(blocks) >= N_NEW // a["dspark_block_size"]
    ids, biased, conf = blocks[0][3]
    assert ids.shape == (1, a["dspark_block_size"] + 1) and biased.shape == (1, a["dspark_block_size"], a["vocab_size"])
