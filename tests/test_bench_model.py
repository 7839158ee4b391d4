"""bench.py's model source (host code, no GPU): the preset's synthetic model by
default, or the tensors of a .glacier / .glrt file given with --model-file."""
import argparse

import numpy as np

import glacier_writer as gw
import glrt_writer as gr


def args(**kw):
    base = dict(model="qwen2.5-0.5b", seed=3, layers=1, model_file=None)
    base.update(kw)
    return argparse.Namespace(**base)


def small():
    from glacier_b200.model import ModelConfig, SyntheticModel
    cfg = ModelConfig(num_layers=1, dim=64, hidden=128, num_heads=4, num_kv_heads=2, head_dim=16, vocab=32, group=16)
    return SyntheticModel(cfg, seed=5)


def test_default_is_the_presets_synthetic_model():
    import bench
    from glacier_b200.model import PRESETS
    cfg, m = bench.bench_model(args())
    assert cfg == PRESETS["qwen2.5-0.5b"] and m.cfg["num_layers"] == 1
    assert bench.data_label(args()) == "synthetic"


def test_model_files(tmp_path):
    import bench
    m = small()
    g = tmp_path / "m.glacier"
    g.write_bytes(bytes(gw.model_image(m)))
    (tmp_path / "m.glacier.json").write_text('{"num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 16}')
    cfg, hm = bench.bench_model(args(model_file=str(g)))
    assert (cfg.dim, cfg.hidden, cfg.num_kv_heads, cfg.group) == (64, 128, 2, 16)
    assert np.array_equal(hm.layers[0]["wd"][0], m.layers[0]["wd"][0])
    assert bench.data_label(args(model_file=str(g))) == "model file m.glacier"
    rng = np.random.default_rng(1)
    emb = (rng.integers(0, 256, 32 * 64 // 2, dtype=np.uint8), (rng.integers(1, 16, 32 * 64 // 16) / 256).astype(np.float32))
    r = tmp_path / "m.glrt"
    r.write_bytes(bytes(gr.build(gr.model_records(m, emb, mlp="pair"), gr.model_cfg(m))))
    cfg, hm = bench.bench_model(args(model_file=str(r)))
    assert cfg.vocab == 32 and np.array_equal(hm.layers[0]["wg"][0], m.layers[0]["wg"][0])


def test_every_rank_decodes_the_same_context_multiset():
    """Weak scaling keeps per-GPU work fixed: each rank's lanes hold the same contexts (rank 0's
    seeded draw from U[ctx_min, ctx_max]) in a rank-specific order."""
    import bench
    a = argparse.Namespace(seed=2024, ctx_min=256, ctx_max=4096)
    r0 = bench.lane_contexts(a, 64, 0)
    assert r0.dtype == np.int32 and r0.min() >= 256 and r0.max() <= 4096
    assert np.array_equal(r0, np.random.default_rng(2024).integers(256, 4097, size=64).astype(np.int32))
    for rank in range(1, 8):
        rk = bench.lane_contexts(a, 64, rank)
        assert np.array_equal(np.sort(rk), np.sort(r0)) and not np.array_equal(rk, r0)
