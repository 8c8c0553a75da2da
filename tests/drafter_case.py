"""The reference's end-to-end lossless scenario (``tests/test_generate_lossless.py:18-86``):
its ``DRAFTER_ARGS``, its order-1 Markov base and prompt (the same numpy draws in the same
order), and a restatement of the greedy speculative loop of ``dspark_mlx/generate.py:39-88``
with ``verify.greedy_accept`` (``verify.py:44-66``), written against the reference's drafter
interface (``forward_spec`` / ``advance``) so that the GPU drafter and the oracle drafter run
in it unchanged.

The reference's drafter starts from MLX's random initialisation, which cannot be reproduced
here; the weights below are seeded draws of the same shapes (the scheme of the block goldens).
The scenario's point is unchanged: whatever the drafts, the emitted stream must equal plain
greedy decoding of the base.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import torch

VOCAB, DIM, N_TARGETS = 32, 16, 2
DRAFTER_ARGS = dict(
    vocab_size=VOCAB, dim=DIM, n_heads=4, head_dim=16, rope_head_dim=8, q_lora_rank=16,
    o_lora_rank=8, o_groups=2, window_size=8, norm_eps=1e-6, rope_theta=10000.0, n_layers=2,
    n_mtp_layers=1, n_routed_experts=4, moe_inter_dim=16, n_activated_experts=2,
    n_shared_experts=1, n_hash_layers=0, score_func="sqrtsoftplus", route_scale=1.5,
    swiglu_limit=10.0, hc_mult=4, hc_sinkhorn_iters=20, dspark_block_size=4,
    dspark_noise_token_id=VOCAB - 1, dspark_target_layer_ids=[0, 1], dspark_markov_rank=8,
    temperature=0.0,
)
MAX_SEQ_LEN = 64
N_NEW = 20


def full_args() -> dict:
    from dsm.config import DSparkArgs

    return dataclasses.asdict(DSparkArgs.from_dict(DRAFTER_ARGS))


def base_and_prompt():
    """``transition [V, V]`` logits, ``embed [V, D * N_TARGETS]`` main hiddens and the 6-token
    prompt: ``default_rng(0)`` drawn in the reference test's order."""
    rng = np.random.default_rng(0)
    transition = rng.standard_normal((VOCAB, VOCAB)).astype(np.float32)
    embed = (rng.standard_normal((VOCAB, DIM * N_TARGETS)) * 0.1).astype(np.float32)
    prompt = rng.integers(0, VOCAB, size=(1, 6)).astype(np.int32)
    return torch.from_numpy(transition), torch.from_numpy(embed), prompt[0].tolist()


def drafter_weights(a: dict, seed: int = 7) -> dict:
    """Every drafter tensor under its reference name (``embed.weight``, ``head.weight``,
    ``blocks.{i}.*``), fp32."""
    g = torch.Generator().manual_seed(seed)
    d, hc, E, inter = a["dim"], a["hc_mult"], a["n_routed_experts"], a["moe_inter_dim"]
    h, hd, ql, og, orank = a["n_heads"], a["head_dim"], a["q_lora_rank"], a["o_groups"], a["o_lora_rank"]
    vocab, rank, mix = a["vocab_size"], a["dspark_markov_rank"], (2 + hc) * hc

    def w(*shape, std, mean=0.0):
        return mean + torch.randn(*shape, generator=g) * std

    t = {"embed.weight": w(vocab, d, std=1.0), "head.weight": w(vocab, d, std=0.5)}
    for i in range(a["n_mtp_layers"]):
        blk = {
            "attn.wq_a.weight": w(ql, d, std=d ** -0.5), "attn.wq_b.weight": w(h * hd, ql, std=ql ** -0.5),
            "attn.wkv.weight": w(hd, d, std=d ** -0.5),
            "attn.wo_a.weight": w(og * orank, h * hd // og, std=(h * hd // og) ** -0.5),
            "attn.wo_b.weight": w(d, og * orank, std=(og * orank) ** -0.5),
            "attn.q_norm.weight": w(ql, std=0.1, mean=1.0), "attn.kv_norm.weight": w(hd, std=0.1, mean=1.0),
            "attn.attn_sink": w(h, std=1.0),
            "ffn.gate.weight": w(E, d, std=0.3), "ffn.gate.bias": w(E, std=0.1),
            "ffn.w1": w(E, inter, d, std=d ** -0.5), "ffn.w3": w(E, inter, d, std=d ** -0.5),
            "ffn.w2": w(E, d, inter, std=inter ** -0.5),
            "ffn.shared_experts.w1.weight": w(inter, d, std=d ** -0.5),
            "ffn.shared_experts.w3.weight": w(inter, d, std=d ** -0.5),
            "ffn.shared_experts.w2.weight": w(d, inter, std=inter ** -0.5),
            "attn_norm.weight": w(d, std=0.1, mean=1.0), "ffn_norm.weight": w(d, std=0.1, mean=1.0),
            "hc_attn_fn": w(mix, hc * d, std=0.05), "hc_ffn_fn": w(mix, hc * d, std=0.05),
            "hc_attn_base": w(mix, std=0.5), "hc_ffn_base": w(mix, std=0.5),
            "hc_attn_scale": w(3, std=1.0), "hc_ffn_scale": w(3, std=1.0),
        }
        if i == 0:
            blk["main_proj.weight"] = w(d, d * len(a["dspark_target_layer_ids"]),
                                        std=(d * len(a["dspark_target_layer_ids"])) ** -0.5)
            blk["main_norm.weight"] = w(d, std=0.1, mean=1.0)
        if i == a["n_mtp_layers"] - 1:
            blk.update({"norm.weight": w(d, std=0.1, mean=1.0),
                        "markov_head.markov_w1.weight": w(vocab, rank, std=0.5),
                        "markov_head.markov_w2.weight": w(vocab, rank, std=0.5),
                        "confidence_head.proj.weight": w(1, d + rank, std=0.05),
                        "hc_head_fn": w(hc, hc * d, std=0.05), "hc_head_base": w(hc, std=0.5),
                        "hc_head_scale": w(1, std=1.0)})
        t.update({f"blocks.{i}.{k}": v.to(torch.float32) for k, v in blk.items()})
    return {k: v.to(torch.float32) for k, v in t.items()}


def plain_greedy(transition: torch.Tensor, start: int, steps: int):
    out, last = [], start
    for _ in range(steps):
        last = int(transition[last].argmax())
        out.append(last)
    return out


def greedy_accept(drafts, base_logits: torch.Tensor):
    """``verify.greedy_accept``: the longest prefix of drafts matching the base argmax, then the
    base argmax at the first divergence (correction or bonus)."""
    base_argmax = base_logits.argmax(dim=-1).tolist()
    n = 0
    while n < len(drafts) and int(drafts[n]) == base_argmax[n]:
        n += 1
    return [int(v) for v in drafts[:n]] + [base_argmax[n]], n


def generate(drafter, transition, embed, prompt, max_new_tokens, device="cpu", on_block=None):
    """``generate.generate`` (b = 1, greedy) against the Markov base. ``on_block(anchor,
    main_hidden, t, out)`` sees every drafted block; returns the emitted tokens."""
    dev = torch.device(device)
    ids = lambda v: torch.tensor([v], dtype=torch.int32, device=dev)  # noqa: E731
    main_hidden = embed[prompt][None].to(dev)          # prefill: [1, L, D * N_TARGETS]
    p1 = transition[prompt[-1]]
    anchor = prompt[-1]
    drafter.forward_spec(ids(anchor), main_hidden, start_pos=0)
    main_hidden = main_hidden[:, -1:].reshape(1, 1, -1)
    t = len(prompt) - 1
    emitted = []
    while len(emitted) < max_new_tokens:
        out = drafter.forward_spec(ids(anchor), main_hidden, start_pos=t)
        if on_block is not None:
            on_block(anchor, main_hidden, t, out)
        d = out[0][0, 1:].cpu().tolist()                # drafts for x_{t+1} .. x_{t+K}
        base_logits = torch.cat([p1[None], transition[d]], dim=0)
        tokens, m = greedy_accept(d, base_logits)
        for j in range(m):
            drafter.advance(embed[d[j]][None].to(dev), t + 1 + j)
        stop = False
        for tok in tokens:
            emitted.append(tok)
            if len(emitted) >= max_new_tokens:
                stop = True
                break
        if stop:
            break
        last = tokens[-1]
        p1 = transition[last]
        main_hidden = embed[last].reshape(1, 1, -1).to(dev)
        t = t + m + 1
        anchor = last
    return emitted
