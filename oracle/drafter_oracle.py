"""CPU oracle for the whole DSpark draft stack (test infrastructure only).

Restates ``DSparkDrafter`` (``dspark_mlx/model/drafter.py:23-54``) from the block oracle:
* ``forward_spec`` (``drafter.py:32-41``): stage 0's ``forward_embed`` (the draft block's
  embeddings and the projected main hidden), every block in order, and on a decode step the
  last block's ``forward_head`` with the shared LM head; the prefill (``start_pos == 0``)
  only seeds the windows;
* ``advance`` (``drafter.py:43-54``): one committed token's main hidden projected by stage 0
  (``main_norm(main_proj(.))``) slides every block's window.
``t`` maps the reference's parameter names to tensors: ``embed.weight``, ``head.weight`` and
``blocks.{i}.<block parameter>`` (the names ``oracle.block_forward`` reads).
"""

from __future__ import annotations

from typing import Dict, List

import torch

from .attention_oracle import KVWindow, linear, rope_tables
from .block_oracle import rms_norm
from .draft_block_oracle import block_advance, block_forward, block_forward_embed, block_forward_head

__all__ = ["OracleDrafter"]


class OracleDrafter:
    def __init__(self, t: Dict[str, torch.Tensor], a: dict, max_seq_len: int = 64):
        self.a = a
        self.embed_w, self.head_w = t["embed.weight"], t["head.weight"]
        self.blocks: List[Dict[str, torch.Tensor]] = []
        for i in range(a["n_mtp_layers"]):
            pre = f"blocks.{i}."
            self.blocks.append({k[len(pre):]: v for k, v in t.items() if k.startswith(pre)})
        self.caches = [KVWindow(a["window_size"]) for _ in self.blocks]
        self.cos, self.sin = rope_tables(a["rope_head_dim"], max_seq_len, a["rope_theta"])

    def forward_spec(self, input_ids: torch.Tensor, main_hidden: torch.Tensor, start_pos: int = 0):
        a = self.a
        h, main_x = block_forward_embed(self.blocks[0], a, main_hidden, input_ids, self.embed_w)
        for bt, cache in zip(self.blocks, self.caches):
            h = block_forward(bt, a, h, start_pos, input_ids, main_x, cache, self.cos, self.sin)
        if start_pos == 0:
            return None
        return block_forward_head(self.blocks[-1], a, h, input_ids, self.head_w, temperature=a["temperature"])

    def advance(self, main_hidden: torch.Tensor, position: int) -> None:
        a, b0 = self.a, self.blocks[0]
        mh = main_hidden.reshape(main_hidden.shape[0], -1)
        main_x = rms_norm(linear(mh, b0["main_proj.weight"]), b0["main_norm.weight"], a["norm_eps"])
        for bt, cache in zip(self.blocks, self.caches):
            block_advance(bt, a, main_x, position, cache, self.cos, self.sin)
