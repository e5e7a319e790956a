"""Right-padding removal on the B200 against the oracle and the reference goldens
(solution/unpad.py:51-72 mask rules, :149-200 metadata, indices, pack, scatter).

The metadata kernels decide validity exactly as the reference's host check does
(binary values, right padding, ignore-index labels on padding, no empty row);
pack and scatter are byte copies, so their outputs must be bit-identical.
"""

from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from tests.helpers import np_of

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "golden_layer_ops.npz")


@pytest.mark.parametrize("case", ["valid", "nonbinary", "leftpad", "labelpad", "empty"])
def test_metadata_matches_reference_rules(case):
    from soupsuck_b200.unpad import pack_batch
    mask = torch.from_numpy(GOLDEN[f"unpad_{case}_mask"]).cuda()
    labels = torch.from_numpy(GOLDEN[f"unpad_{case}_labels"]).cuda()
    expected = tuple(int(x) for x in GOLDEN[f"unpad_{case}_lengths"])
    if not expected:
        with pytest.raises(ValueError):
            pack_batch(mask, labels)
        return
    pb = pack_batch(mask, labels)
    assert pb.lengths == expected
    assert np_of(pb.cu_seqlens).tolist() == [0, *np.cumsum(expected).tolist()]


@pytest.mark.parametrize("dtype", [torch.bool, torch.int32, torch.float16, torch.float32])
def test_metadata_mask_dtypes(dtype):
    from soupsuck_b200.unpad import pack_batch
    mask = torch.from_numpy(GOLDEN["unpad_valid_mask"]).cuda().to(dtype)
    assert pack_batch(mask).lengths == tuple(int(x) for x in GOLDEN["unpad_float_lengths"])


def test_pack_scatter_bits_and_gradients():
    from soupsuck_b200.unpad import pack, pack_batch, scatter
    mask = torch.from_numpy(GOLDEN["unpad_valid_mask"]).cuda()
    pb = pack_batch(mask)
    x = torch.from_numpy(GOLDEN["unpad_valid_x"]).cuda().requires_grad_()
    packed = pack(x, pb)
    assert np.array_equal(np_of(packed), GOLDEN["unpad_valid_packed"][0])
    back = scatter(packed, pb)
    assert np.array_equal(np_of(back), GOLDEN["unpad_valid_scattered"])
    g = torch.randn_like(back)
    back.backward(g)
    ref = O.unpad_scatter(O.unpad_pack(np_of(g), pb.lengths), pb.lengths, pb.sequence)
    assert np.array_equal(np_of(x.grad), ref)


@pytest.mark.parametrize("rows,seq,width", [(4, 512, 1536), (64, 33, 7), (3, 2048, 3584)])
def test_pack_scatter_random_batches(rows, seq, width):
    from soupsuck_b200.unpad import pack, pack_batch, scatter
    rng = np.random.default_rng(rows * seq)
    lengths = rng.integers(1, seq + 1, size=rows)
    mask = (np.arange(seq)[None, :] < lengths[:, None]).astype(np.int64)
    labels = np.where(mask == 1, 5, -100)
    pb = pack_batch(torch.from_numpy(mask).cuda(), torch.from_numpy(labels).cuda())
    assert pb.lengths == tuple(int(x) for x in lengths)
    x = torch.randn((rows, seq, width), device="cuda").half()
    packed = pack(x, pb)
    assert np.array_equal(np_of(packed), O.unpad_pack(np_of(x), pb.lengths))
    back = scatter(packed, pb)
    assert np.array_equal(np_of(back), O.unpad_scatter(np_of(packed), pb.lengths, seq))
