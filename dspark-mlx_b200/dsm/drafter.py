"""The whole DSpark draft stack on the GPU: ``DSparkDrafter`` (``dspark_mlx/model/drafter.py:23-54``).

Same constructor (``DSparkDrafter(args, max_seq_len)``), calls and parameter names as the
reference, so a decode loop written against the reference's drafter (``generate.py:39-88``)
drives this one unchanged:
* ``embed.weight [vocab, dim]`` and ``head.weight [vocab, dim]``, shared by the blocks;
* ``blocks``: ``n_mtp_layers`` :class:`dsm.draft_block.DSparkBlock`, stage ``i`` each;
* ``forward_spec(input_ids, main_hidden, start_pos)`` (``drafter.py:32-41``): stage 0 embeds
  the draft block and projects the main hidden, every block runs in order; the prefill
  (``start_pos == 0``) seeds the windows and returns ``None``, a decode step returns the
  last block's ``forward_head``: ``(output_ids [b, K+1], biased logits [b, K, vocab],
  confidence [b, K])``;
* ``advance(main_hidden, position)`` (``drafter.py:43-54``): one committed token's main
  hidden, projected once by stage 0, slides every block's window.

Every step runs on ``libdsm`` kernels through the blocks; CPU tensors are rejected.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import nn

from .config import DSparkArgs
from .draft_block import DSparkBlock


class _Table(nn.Module):
    """A ``weight [rows, dim]`` holder under the reference's module names (``embed``, ``head``)."""

    def __init__(self, rows: int, dim: int):
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(rows, dim, dtype=torch.float32), requires_grad=False)


class DSparkDrafter(nn.Module):
    def __init__(self, args, max_seq_len: int = 8192):
        super().__init__()
        if isinstance(args, dict):
            args = DSparkArgs.from_dict(args)
        self.n_mtp_layers = args.n_mtp_layers
        self.block_size = args.dspark_block_size
        self.embed = _Table(args.vocab_size, args.dim)
        self.head = _Table(args.vocab_size, args.dim)
        self.blocks = nn.ModuleList(DSparkBlock(args, i, max_seq_len) for i in range(args.n_mtp_layers))

    def forward_spec(self, input_ids: torch.Tensor, main_hidden: torch.Tensor,
                     start_pos: int = 0) -> Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
        h, main_x = self.blocks[0].forward_embed(main_hidden, input_ids, self.embed)
        for blk in self.blocks:
            h = blk(h, start_pos, input_ids, main_x)
        if start_pos == 0:
            return None
        return self.blocks[-1].forward_head(h, input_ids, self.head)

    def advance(self, main_hidden: torch.Tensor, position: int) -> None:
        mh = main_hidden.reshape(main_hidden.shape[0], -1)
        main_x = self.blocks[0].project_main(mh)
        for blk in self.blocks:
            blk.advance(main_x, position)
