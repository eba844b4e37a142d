"""Pin the torch restatement (used by the full-size GPU checks) on CPU."""
import os

import numpy as np
import pytest
import torch

from oracle import holonomy_oracle as O
from oracle import torch_ref
from test_oracle import case_inputs, load


@pytest.mark.parametrize("name", ["tiny_es01", "tiny_es15", "d48_L40", "bf16_d48_L64"])
def test_torch_ref_vs_golden(name):
    z = load(name)
    sd, x, H, es = case_inputs(z)
    x = torch.from_numpy(x)
    y64 = torch_ref.module_forward(sd, x, H, es, dtype=torch.float64, batch_slice=1).numpy()
    assert O.rel_l2(y64, z["y_chunked_f64"]) < 1e-11
    y32 = torch_ref.module_forward(sd, x, H, es, dtype=torch.float32, batch_slice=2).numpy()
    assert O.rel_l2(y32, z["y_chunked_f64"]) < 1e-5


def test_torch_ref_head_groups_equal_all_heads():
    """The head-group option (used to bound memory at configs[4]) gives the all-heads result:
    heads are independent between the qkv split and the out projection."""
    z = load("d48_L40")
    sd, x, H, es = case_inputs(z)
    x = torch.from_numpy(x)
    y_all = torch_ref.module_forward(sd, x, H, es, dtype=torch.float64, batch_slice=1).numpy()
    for hg in (1, 3):
        y = torch_ref.module_forward(sd, x, H, es, dtype=torch.float64, batch_slice=1,
                                     head_group=hg).numpy()
        assert O.rel_l2(y, y_all) < 1e-14
