"""Seeded GPT init reproduces the reference's parameters exactly (CPU, no kernels).

The golden state dicts come from the reference's own GPT(**cfg) under the same
seed (tests/golden/gen_golden.py), so equal tensors mean the module tree,
parameter names, registration order and init rules all match
(model/gpt.py:11-90, model/utils.py:5-37)."""
import os

import pytest
import torch

from rgpt_b200.model import GPT

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("tag", ["gpt", "rgpt", "elastic"])
def test_seeded_init_matches_reference_state_dict(tag):
    g = torch.load(os.path.join(GOLD, f"model_{tag}.pt"), weights_only=False)
    torch.manual_seed(g["seed"])
    model = GPT(**g["cfg"])
    ours = model.state_dict()
    ref = g["state"]
    assert set(ours.keys()) == set(ref.keys())
    for k, v in ref.items():
        assert ours[k].shape == v.shape, k
        assert torch.equal(ours[k], v), k


def test_parameter_groups_match_trainer_rules():
    from oracle.ref_ops import param_groups
    from rgpt_b200.optimizer import trainer_param_groups
    g = torch.load(os.path.join(GOLD, "model_rgpt.pt"), weights_only=False)
    model = GPT(**g["cfg"])
    ours = trainer_param_groups(model, tie_word_embeddings=False)
    muon, dec, nodec = param_groups(list(model.named_parameters()))
    names = {id(p): n for n, p in model.named_parameters()}
    assert [names[id(p)] for p in ours[0]["params"]] == muon
    assert [names[id(p)] for p in ours[1]["params"]] == dec
    assert [names[id(p)] for p in ours[2]["params"]] == nodec
