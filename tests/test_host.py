"""Host-side logic without a GPU: synthetic inputs, the safetensors writer/reader and the
layout plan (the reference's TestStreamer/TestGraph, Opure_TestHarness.cpp:147-322, on a
synthetic model since the real checkpoint is not available)."""
import json
import math
import os

import numpy as np
import pytest

import oracle
from golden.make_golden import Rng
from voxelengine import cuda as cu
from voxelengine import engine as ve

TINY = dict(vocab=512, hidden=128, inter=256, layers=2, heads=2, kv_heads=1, max_pos=256)


@pytest.fixture(scope="module")
def tiny_dir(tmp_path_factory):
    return ve.synth_model(str(tmp_path_factory.mktemp("tiny")), seed=11, **TINY)


def test_prompt_is_rng_mod_vocab():
    r = Rng(1)
    want = [r.next_u32() % 49152 for _ in range(32)]
    assert list(ve.prompt(1, 49152, 32)) == want


def test_permutation_is_fisher_yates():
    n = 97
    r = Rng(3)
    p = list(range(n))
    for i in range(n, 1, -1):
        j = r.next_u32() % i
        p[i - 1], p[j] = p[j], p[i - 1]
    got = ve.permutation(3, n)
    assert list(got) == p and sorted(got) == list(range(n))


def test_uniforms():
    r = Rng(9)
    want = np.array([r.next_u32() / 4294967296.0 for _ in range(100)], np.float32)
    assert np.array_equal(ve.uniforms(9, 100), want)


def test_spec_uniform_streams():
    # The speculative loop's per-sequence streams: the oracle's restatement and the
    # engine's Rng draw the same uniforms from seed ^ s * 0x9E3779B97F4A7C15.
    from oracle import spec
    for seed, s in ((0, 0), (3, 1), (12, 15)):
        derived = seed ^ ((s * spec.GOLDEN) & spec.MASK)
        r = spec.Rng(derived)
        assert np.array_equal(np.array([r.uniform() for _ in range(64)], np.float32),
                              ve.uniforms(derived, 64))


def test_normals_box_muller():
    r = Rng(5)
    want = []
    for _ in range(50):
        u1 = (r.next_u32() + 0.5) / 4294967296.0
        u2 = (r.next_u32() + 0.5) / 4294967296.0
        rad = math.sqrt(-2.0 * math.log(u1))
        want += [rad * math.cos(2 * math.pi * u2), rad * math.sin(2 * math.pi * u2)]
    want = oracle.f32_to_f16(np.array(want, np.float32) * np.float32(0.02))
    assert np.array_equal(ve.normal_f16(5, 0.02, 100), want)


def test_synth_model_layout(tiny_dir):
    cfg = json.load(open(os.path.join(tiny_dir, "config.json")))
    assert cfg["num_key_value_heads"] == 1 and cfg["tie_word_embeddings"] is True
    t = oracle.read_safetensors(os.path.join(tiny_dir, "model.safetensors"))
    assert t["model.embed_tokens.weight"][1] == [512, 128]
    assert t["model.layers.1.self_attn.k_proj.weight"][1] == [64, 128]
    assert t["model.layers.0.mlp.down_proj.weight"][1] == [128, 256]
    assert np.all(t["model.norm.weight"][2] == 0x3C00)  # gains are 1.0
    # The embedding is the first 512*128 draws of the weight stream.
    emb = np.asarray(t["model.embed_tokens.weight"][2]).ravel()
    assert np.array_equal(emb, ve.normal_f16(11, 0.02, emb.size))


def test_synth_int8_and_draft(tmp_path):
    d = ve.synth_model(str(tmp_path / "q"), seed=11, int8=True, **TINY)
    t = oracle.read_safetensors(os.path.join(d, "model.safetensors"))
    dt, _, q, s = t["model.layers.0.self_attn.q_proj.weight"]
    assert dt == "I8" and 0 < s < 1 and np.abs(q).max() == 127
    base = oracle.read_safetensors(os.path.join(ve.synth_model(str(tmp_path / "f"), seed=11, **TINY),
                                                "model.safetensors"))
    f = oracle.f16_to_f32(np.asarray(base["model.layers.0.self_attn.q_proj.weight"][2]))
    assert np.abs(q * s - f).max() <= s / 2 + 1e-7
    dr = ve.synth_model(str(tmp_path / "d"), seed=11, noise_seed=6, noise_std=0.004, **TINY)
    td = oracle.read_safetensors(os.path.join(dr, "model.safetensors"))
    g = oracle.f16_to_f32(np.asarray(td["model.layers.0.self_attn.q_proj.weight"][2]))
    diff = g - f
    assert 0.003 < diff.std() < 0.005  # N(0, 0.004) perturbation


def test_inspect_plans_layout(tiny_dir):
    info = ve.inspect(tiny_dir)
    assert (info.vocab, info.hidden, info.layers, info.head_dim) == (512, 128, 2, 64)
    assert info.w_dtype == cu.W_F16
    # Streamed bytes per step: every matrix once in fp16 + gains + the tied lm_head.
    h, ff = 128, 256
    per_layer = ((2 * 64 + 2 * 64) * h + h * h + 3 * ff * h) * 2 + 2 * h * 2
    assert info.stream_bytes == 2 * per_layer + 512 * h * 2 + h * 2
    assert info.kv_bytes_per_token == 2 * 2 * 1 * 64 * 2


def test_inspect_smollm_shape_bytes(tmp_path):
    # Only config + header matter for planning: write the SmolLM-135M geometry with a
    # 1-layer file and check the per-layer byte accounting used by the roofline.
    d = ve.synth_model(str(tmp_path / "s"), seed=0, layers=1)
    info = ve.inspect(d)
    assert info.stream_bytes == 7077888 + 2 * 576 * 2 + 56623104 + 576 * 2


@pytest.mark.parametrize("edit,reason", [
    (lambda c: c.update(hidden_act="gelu"), "hidden_act"),
    (lambda c: c.update(num_attention_heads=4), "head_dim"),
    (lambda c: c.update(attention_bias=True), "bias"),
    (lambda c: c.update(num_key_value_heads=3, num_attention_heads=4), "divisible"),
])
def test_inspect_refuses_unsupported(tiny_dir, tmp_path, edit, reason):
    cfg = json.load(open(os.path.join(tiny_dir, "config.json")))
    edit(cfg)
    d = tmp_path / "m"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(cfg))
    os.symlink(os.path.join(tiny_dir, "model.safetensors"), d / "model.safetensors")
    with pytest.raises(cu.OpureError) as e:
        ve.inspect(str(d))
    assert reason in str(e.value)


def test_inspect_rejects_shape_mismatch(tiny_dir, tmp_path):
    cfg = json.load(open(os.path.join(tiny_dir, "config.json")))
    cfg["intermediate_size"] = 512
    d = tmp_path / "m"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(cfg))
    os.symlink(os.path.join(tiny_dir, "model.safetensors"), d / "model.safetensors")
    with pytest.raises(cu.OpureError) as e:
        ve.inspect(str(d))
    assert "gate_proj" in str(e.value)


def test_truncated_safetensors_is_refused(tiny_dir, tmp_path):
    d = tmp_path / "t"
    d.mkdir()
    (d / "config.json").write_text(open(os.path.join(tiny_dir, "config.json")).read())
    raw = open(os.path.join(tiny_dir, "model.safetensors"), "rb").read()
    (d / "model.safetensors").write_bytes(raw[: len(raw) - 1000])
    with pytest.raises(cu.OpureError) as e:
        ve.inspect(str(d))
    assert "beyond the file" in str(e.value)


def test_synth_kv_matches_splitmix_restatement():
    # The seeded long-context KV values (host form of opure_kv_synth) against an
    # independent restatement of SplitMix64 + fp16(4u - 2).
    M = (1 << 64) - 1

    def splitmix(x):
        z = (x + 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        return z ^ (z >> 31)

    seed, slot, L, H, T, D = 5, 3, 2, 2, 9, 64
    got = ve.synth_kv(seed, slot, L, H, T, D)
    want = np.empty((L, 2, H, T, D), np.float16)
    for idx in np.ndindex(L, 2, H, T, D):
        l, s, h, t, d = idx
        i = (((l * 2 + s) * H + h) * 65536 + t) * D + d
        u = np.float32(splitmix(seed ^ (slot << 48) ^ i) >> 40) / np.float32(16777216.0)
        want[idx] = np.float16(u * np.float32(4) - np.float32(2))
    assert np.array_equal(got, want.view(np.uint16))
