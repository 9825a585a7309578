"""Shared helpers for the GPU parity tests."""

import numpy as np
import pytest
import torch

from oracle import tree as ot
from retree_b200 import synthetic


def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


def random_tree(seed, budget, max_depth=16):
    parents = synthetic.random_tree_parents(seed, budget, max_depth=max_depth).tolist()
    vis = ot.visibility(parents)
    return parents, vis


def bits_tensor(vis, device, words=None):
    return torch.from_numpy(ot.pack_bits(vis, words).view(np.int32)).to(device)
