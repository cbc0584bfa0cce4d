"""SabreKVCache semantics (host tensors; no kernel involved)."""

import torch

from sabrecoder_b200.kv_cache import SabreKVCache


def test_update_slots_advance_crop():
    c = SabreKVCache(num_layers=2, num_kv_heads=2, head_dim=4, max_cache_len=10, device="cpu",
                     dtype=torch.float32)
    k = torch.arange(2 * 3 * 4, dtype=torch.float32).view(1, 2, 3, 4)
    kk, vv = c.update(k, k + 1, 0)
    assert kk.shape == (1, 2, 3, 4) and torch.equal(kk, k) and torch.equal(vv, k + 1)
    assert c.get_seq_length(0) == 3 and c.get_seq_length(1) == 0
    kb, vb, pos = c.slots(1, 4)
    assert pos == 0 and kb.shape[2] == 10
    kb[:, :, :4] = 7.0
    kk, _ = c.advance(1, 4)
    assert kk.shape[2] == 4 and (kk == 7.0).all()
    c.crop(2)
    assert c.get_seq_length(0) == 2 and c.get_seq_length(1) == 2
    assert c.get_mask_sizes(5, 0) == (7, 0)
    assert c.max_cache_len == 10 and c.max_batch_size == 1
    try:
        c.update(torch.zeros(1, 2, 9, 4), torch.zeros(1, 2, 9, 4), 0)
    except ValueError as e:
        assert "full" in str(e)
    else:
        raise AssertionError("overflow not detected")
    c.reset()
    assert c.get_seq_length() == 0
