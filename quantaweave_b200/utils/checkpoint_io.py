"""The single place where checkpoints are unpickled (reference ``src/checkpoint_io.py``).

Checkpoints (``model.pt``, ``model.rank{r}.pt``, ``adapter.pt``, ``model.int{b}.pt``) are ``torch.save``'d dicts
that mix tensors with Python objects (RNG state, configs, optimizer state), so loading needs
``weights_only=False``, which is equivalent to ``pickle.load``: only load checkpoints you produced or trust.
"""

from __future__ import annotations

from pathlib import Path
from typing import Optional, Union

import torch


def load_checkpoint(path: Union[str, Path], map_location: Optional[Union[str, torch.device]] = None) -> dict:
    return torch.load(path, map_location=map_location, weights_only=False)
