"""GPU: PiZeroRunner contract (port of the reference's python/tests/test_pizero_runner.py, on the
`cuda` target with float16 instead of the `c` target with float32)."""

import numpy as np
import pytest

from conftest import cosine
from tests.golden import recipes

pytestmark = pytest.mark.gpu

DUMMY_KWARGS = dict(recipes.DUMMY, dtype="float16")


@pytest.fixture(scope="module")
def runner():
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.sample import PiZeroRunner

    return PiZeroRunner(Pi0Config(**DUMMY_KWARGS), target="cuda")


@pytest.fixture
def loaded(runner):
    rng = np.random.default_rng(0)
    arrays = []
    for _name, p in runner.named_params:
        shape = [int(s) for s in p.shape]
        if p.dtype.startswith(("int", "uint")):
            arrays.append(np.zeros(shape, p.dtype))
        else:
            arrays.append((0.02 * rng.standard_normal(shape)).astype(p.dtype))
    params = runner.to_params(arrays)
    cfg = runner.config
    prefix = (0.02 * rng.standard_normal((1, cfg.prefix_len, cfg.vlm.width))).astype("float32")
    return params, prefix


def test_cublas_guard_off(runner):
    assert runner.cublas is False


def test_sample_output_shape_and_finite(runner, loaded):
    params, prefix = loaded
    cfg = runner.config
    out = runner.sample(params, prefix, num_steps=cfg.num_denoise_steps, seed=7)
    assert out.shape == (1, cfg.action_horizon, cfg.action_dim)
    assert out.dtype == np.float32
    assert np.all(np.isfinite(out))


def test_sample_graph_matches_host_loop(runner, loaded):
    params, prefix = loaded
    cfg = runner.config
    noise = np.random.default_rng(3).standard_normal(
        (1, cfg.action_horizon, cfg.action_dim)).astype("float32")
    host = runner.sample(params, prefix, noise=noise, num_steps=cfg.num_denoise_steps)
    graph = runner.sample_graph(params, prefix, noise=noise)
    assert graph.shape == host.shape == (1, cfg.action_horizon, cfg.action_dim)
    assert cosine(host, graph) >= 0.99999


def test_sample_accepts_prefix_pad(runner, loaded):
    params, prefix = loaded
    cfg = runner.config
    pad = np.zeros((cfg.prefix_len,), dtype=np.float32)
    pad[: cfg.prefix_len // 2] = 1.0
    out = runner.sample(params, prefix, num_steps=cfg.num_denoise_steps, seed=1, prefix_pad=pad)
    assert out.shape == (1, cfg.action_horizon, cfg.action_dim)
    assert np.all(np.isfinite(out))


def test_vm_function_contract(runner, loaded):
    """test_compile_and_run.py: every exported function through the VM-style interface."""
    from mlc_vla.sample import make_prefix_mask_np, make_rope_np, make_time_embs

    params, prefix = loaded
    cfg = runner.config
    vm = runner.vm
    rng = np.random.default_rng(1)
    pm = make_prefix_mask_np(cfg.prefix_len)
    c, s = make_rope_np(cfg.suffix_len, cfg.vlm.head_dim, cfg.rope_theta, offset=cfg.prefix_len)
    kv = vm["prefill"](prefix.astype(np.float16), pm, params)
    keys, values = kv[0], kv[1]
    assert cfg.prefix_len in keys.shape and cfg.vlm.head_dim in keys.shape
    assert np.all(np.isfinite(keys.numpy())) and np.all(np.isfinite(values.numpy()))
    x_t = rng.standard_normal((1, cfg.action_horizon, cfg.action_dim)).astype(np.float16)
    te = rng.standard_normal((1, cfg.action_expert.width)).astype(np.float16)
    v = vm["denoise_step_kv"](keys, values, x_t, te, c, s, pm, params).numpy()
    assert v.shape == (1, cfg.action_horizon, cfg.action_dim) and str(v.dtype) == "float32"
    x0 = rng.standard_normal((1, cfg.action_horizon, cfg.action_dim)).astype(np.float32)
    tes = np.concatenate(make_time_embs(cfg.num_denoise_steps, cfg.action_expert.width), 0)
    out = vm["denoise_loop_kv"](keys, values, x0, tes.astype(np.float16), c, s, pm, params).numpy()
    assert out.shape == (1, cfg.action_horizon, cfg.action_dim) and np.all(np.isfinite(out))


def test_cached_tables_follow_the_pad_pattern(runner, loaded):
    """The runner keeps the pad mask, suffix RoPE tables and time embeddings on the device, keyed
    by the pad pattern: alternating patterns give each pattern's own result, identical to a
    fresh runner's (the tables are recomputed there)."""
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.sample import PiZeroRunner

    params, prefix = loaded
    cfg = runner.config
    noise = np.random.default_rng(5).standard_normal(
        (1, cfg.action_horizon, cfg.action_dim)).astype("float32")
    pad_a = np.ones((cfg.prefix_len,), np.float32)
    pad_a[-100:] = 0.0
    pad_b = np.ones((cfg.prefix_len,), np.float32)
    pad_b[300:400] = 0.0
    outs = [runner.sample_graph(params, prefix, noise=noise, prefix_pad=p)
            for p in (pad_a, pad_b, None, pad_a)]
    assert np.array_equal(outs[0], outs[3])
    assert not np.array_equal(outs[0], outs[1]) and not np.array_equal(outs[0], outs[2])
    fresh = PiZeroRunner(Pi0Config(**DUMMY_KWARGS), target="cuda")
    fparams = fresh.to_params(list(params))
    assert np.array_equal(fresh.sample_graph(fparams, prefix, noise=noise, prefix_pad=pad_b),
                          outs[1])


def test_sample_graph_from_pinned_host_buffers(runner, loaded):
    """The pinned-prefix upload and the staged noise upload are asynchronous: results equal the
    device-resident call bit for bit, a pinned buffer rewritten right after a call returns does
    not leak into that call, and the table buffers follow a change of pad pattern."""
    import torch

    params, prefix = loaded
    cfg = runner.config
    rng = np.random.default_rng(11)
    noises = [rng.standard_normal((1, cfg.action_horizon, cfg.action_dim)).astype("float32")
              for _ in range(2)]
    prefixes = [prefix, (prefix + 0.01 * rng.standard_normal(prefix.shape)).astype("float32")]
    want = [runner.sample_graph(params, torch.from_numpy(p).cuda(), noise=n)
            for p, n in zip(prefixes, noises)]
    pinned = torch.from_numpy(prefixes[0].copy()).pin_memory()
    for i in range(2):
        got = runner.sample_graph(params, pinned, noise=noises[i])
        np.testing.assert_array_equal(got, want[i])
        pinned.copy_(torch.from_numpy(prefixes[1]))  # next call's prefix, written at once
    pad = np.ones((cfg.prefix_len,), np.float32)
    pad[-3:] = 0
    padded = runner.sample_graph(params, pinned, noise=noises[1], prefix_pad=pad)
    again = runner.sample_graph(params, pinned, noise=noises[1])
    np.testing.assert_array_equal(again, want[1])
    assert not np.array_equal(padded, want[1])
