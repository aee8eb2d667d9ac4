"""On-disk cache of packed expert tiers (CPU): a bank written by
``ExpertBank.save`` loads back byte for byte with the same expert map."""
import torch

from exq_b200.experts import ExpertBank


def _fake_bank():
    h, i = 256, 128
    g = torch.Generator().manual_seed(0)
    b = ExpertBank(hidden=h, inter=i, act_dtype=torch.bfloat16, n_routed=3, n_shared=1,
                   tiers=["INT4", "BF16", "INT4", "INT8"])
    b.storage["INT4"] = (torch.randint(0, 255, (2, 2 * i, h // 2), dtype=torch.uint8, generator=g),
                         torch.randn(2, h // 128, 2 * i, generator=g).half(),
                         torch.randint(0, 255, (2, h, i // 2), dtype=torch.uint8, generator=g),
                         torch.randn(2, i // 128, h, generator=g).half())
    b.storage["BF16"] = (torch.randn(1, 2 * i, h, generator=g).half(), None,
                         torch.randn(1, h, i, generator=g).half(), None)
    b.storage["INT8"] = (torch.randint(-127, 127, (1, 2 * i, h), dtype=torch.int8, generator=g),
                         torch.randn(1, 2 * i, generator=g).half(),
                         torch.randint(-127, 127, (1, h, i), dtype=torch.int8, generator=g),
                         torch.randn(1, h, generator=g).half())
    b.index = {"INT4": [0, 2], "BF16": [1], "INT8": [3]}
    b._finalize(torch.device("cpu"))
    return b


def test_bank_cache_round_trip(tmp_path):
    b = _fake_bank()
    path = tmp_path / "layer0.pt"
    b.save(path)
    c = ExpertBank.load(path, device="cpu")
    assert (c.hidden, c.inter, c.n_routed, c.n_shared, c.act_dtype) == \
        (b.hidden, b.inter, b.n_routed, b.n_shared, b.act_dtype)
    assert c.tiers == b.tiers and c.index == b.index
    assert torch.equal(c.expert_slot, b.expert_slot)
    for name, st in b.storage.items():
        for x, y in zip(st, c.storage[name]):
            assert (x is None and y is None) or torch.equal(x, y)
    assert c.cstruct.n_tier[0] == 1 and c.cstruct.n_tier[1] == 1 and c.cstruct.n_tier[2] == 2


def test_bank_cache_rejects_other_files(tmp_path):
    import pytest
    path = tmp_path / "x.pt"
    torch.save({"version": 99}, path)
    with pytest.raises(ValueError):
        ExpertBank.load(path, device="cpu")
