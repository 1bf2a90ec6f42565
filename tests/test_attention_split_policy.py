"""The paged-attention split policy, checked without a GPU through the host-only
opure_attention_scratch_bytes (the scratch holds one (m, l, acc[hd]) partial per query
entry, kv head and split, then one counter per entry and kv head).

The policy for head_dim 64 / 128 was set from a B200 sweep of split sizes: splits are
multiples of 128 tokens; about one wave of three CTAs per SM (148 SMs), at most 32 splits;
splits of at most 3072 tokens instead when that turns a grid of fewer than three waves into
three or more. These cases pin the split counts the sweep chose.

The policy reads the current device's SM count (148 with no visible device): on a device
with another count the pinned numbers do not apply and the module is skipped.
"""
import pytest

from voxelengine import cuda as cu


def _visible_sm_count():
    try:
        import torch
        if torch.cuda.is_available():
            return torch.cuda.get_device_properties(0).multi_processor_count
    except Exception:
        pass
    return None


_SMS = _visible_sm_count()
pytestmark = pytest.mark.skipif(_SMS not in (None, 148), reason=f"split counts pinned for 148 SMs, device has {_SMS}")


def scratch(entries_kv, splits, G, hd=64):
    part = entries_kv * splits * G * (hd + 2) * 4
    return ((part + 255) // 256) * 256 + entries_kv * 4


@pytest.mark.parametrize("B,ctx,splits", [
    (64, 32768, 11),   # 192 pairs: splits of 3072 tokens give 4.8 waves
    (64, 8192, 2),     # 3 splits would be 1.3 waves: stay at one wave
    (8, 32768, 19),    # 24 pairs: one wave
    (1, 32768, 32),    # capped: the last CTA merges every split
    (1, 8192, 32),
    (64, 168, 1),      # decode lengths: one split of 256 tokens
])
def test_config1_split_counts(B, ctx, splits):
    assert cu.attention_scratch_bytes(B, 1, 9, 3, 64, ctx) == scratch(B * 3, splits, 3)


def test_large_model_keeps_one_split():
    # 64 sequences x 32 kv heads already fill more than three waves without splitting.
    assert cu.attention_scratch_bytes(64, 1, 32, 32, 64, 4160) == scratch(64 * 32, 1, 1)


def test_requested_split_rounds_to_128_tokens():
    assert cu.attention_scratch_bytes(2, 1, 8, 8, 128, 1500, 100) == scratch(16, 12, 1, hd=128)
