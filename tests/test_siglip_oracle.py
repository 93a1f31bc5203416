"""The SigLIP oracle (``embed_image``) against transformers' SigLIP outputs committed by
``tests/golden/make_siglip_golden.py``, and the vision stage's parameter table against the
reference loader's own name map (``tests/golden/loader_map.json``)."""

import json
import os

import numpy as np

from conftest import ROOT, cosine, max_abs
from oracle import pi0_oracle as O
from oracle import siglip_oracle as S
from tests.golden import make_siglip_golden as G


def _golden():
    return dict(np.load(G.PATH))


def test_vision_table_matches_reference_loader_map():
    from mlc_vla.model.pi0 import Pi0Config
    from mlc_vla.model.pi0.pi0_model import vision_named_params

    names = [n for n, _ in vision_named_params(Pi0Config())]
    with open(os.path.join(ROOT, "tests", "golden", "loader_map.json")) as f:
        ref = json.load(f)["full"]
    assert set(names) == {k for k in ref if k.startswith("vision.")}
    assert len(names) == len(set(names)) == 3 + 16 * 27 + 4


def test_oracle_matches_transformers_mini():
    g = _golden()
    cfg = G.configs()["mini"]
    from mlc_vla.model.pi0.pi0_model import vision_named_params

    p = O.prepare_params(O.random_params(vision_named_params(cfg), seed=0), "float32")
    image = G.inputs(cfg, batch=2)
    assert np.isclose(float(np.sum(image, dtype=np.float64)), float(g["mini_image_sum"]))
    out = S.embed_image(p, cfg, image)
    assert cosine(out, g["mini_out"]) >= 0.99999 and max_abs(out, g["mini_out"]) < 1e-5


def test_oracle_matches_transformers_wide():
    """So400m widths (hidden 1152, 16 heads of 72, MLP 4304, 256 patches), one layer."""
    g = _golden()
    cfg = G.configs()["wide"]
    from mlc_vla.model.pi0.pi0_model import vision_named_params

    p = O.prepare_params(O.random_params(vision_named_params(cfg), seed=0), "float32")
    image = G.inputs(cfg, batch=1)
    assert np.isclose(float(np.sum(image, dtype=np.float64)), float(g["wide_image_sum"]))
    out = S.embed_image(p, cfg, image)
    rows = out[:, G.ROWS]
    assert cosine(rows, g["wide_rows"]) >= 0.99999 and max_abs(rows, g["wide_rows"]) < 1e-5
    l2 = np.sqrt(np.sum(out.astype(np.float64) ** 2, axis=-1))
    np.testing.assert_allclose(l2, g["wide_row_l2"], rtol=1e-5)


def test_patchify_order():
    """Patch (py, px) row = image rows py·p .. py·p+p-1, columns px·p .., flattened (row, col,
    channel): the reference's _patchify (siglip.py:104-114)."""
    img = np.arange(2 * 28 * 28 * 3, dtype=np.float32).reshape(2, 28, 28, 3)
    x = S.patchify(img, 14)
    assert x.shape == (2, 4, 14 * 14 * 3)
    b, py, px, i, j, c = 1, 1, 0, 3, 5, 2
    assert x[b, py * 2 + px, (i * 14 + j) * 3 + c] == img[b, py * 14 + i, px * 14 + j, c]
