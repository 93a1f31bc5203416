"""GPU: ``embed_language`` (reference ``pi0_model.py:101-104``: embedding gather · sqrt(width),
spec ``:217-220``) through ``pi0_embed_language``, bit-exact against the oracle's restatement,
at the PaliGemma vocabulary and width (257152 × 2048) and on a small table."""

import numpy as np
import pytest

from oracle import pi0_oracle as O

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("vocab,width,dtype", [(257_152, 2048, torch.float16),
                                               (1000, 256, torch.bfloat16),
                                               (300, 64, torch.float16)])
def test_embed_language_bit_exact(vocab, width, dtype):
    from mlc_vla.runtime import embed_language

    g = torch.Generator(device="cuda").manual_seed(vocab + width)
    table = torch.randn((vocab, width), generator=g, device="cuda").to(dtype)
    rng = np.random.default_rng(1)
    ids = rng.integers(0, vocab, size=(1, 200)).astype(np.int32)
    ids[0, :3] = [0, vocab - 1, 7]
    out = embed_language(table, ids)
    torch.cuda.synchronize()
    assert out.shape == (1, 200, width) and out.dtype == dtype
    uniq = np.unique(ids)
    rows = table[torch.from_numpy(uniq).long().cuda()].float().cpu().numpy()
    remap = {int(v): i for i, v in enumerate(uniq)}
    ref_dt = "float16" if dtype == torch.float16 else "bfloat16"
    want = O.embed_language(rows, np.vectorize(remap.get)(ids), ref_dt)
    got = out.float().cpu().numpy().reshape(-1, width)
    assert np.array_equal(got, np.asarray(want, np.float32).reshape(-1, width))


def test_embed_language_rejects_out_of_range_ids():
    from mlc_vla.runtime import embed_language

    table = torch.randn((50, 64), device="cuda").half()
    with pytest.raises(ValueError):
        embed_language(table, np.array([[1, 2, 50]], np.int32))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = embed_language(table, np.array([[1, -1, 3]], np.int32), err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    assert torch.count_nonzero(out[0, 1]).item() == 0
    assert torch.count_nonzero(out[0, 0]).item() > 0
