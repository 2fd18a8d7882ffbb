"""Row shards of a product equal the same rows of the unsharded product (needs a GPU).

Each shard runs on its own Simulator, as each rank of a multi-GPU job does, so
this checks the vector offsets that keep noise addresses global.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import memfast_b200

    return memfast_b200


def _config(mf, **effects):
    return mf.Config(array_size=(128, 128), rows_per_read=32, weight_quant_gran=(32, 1), input_quant_gran=(1, 32),
                     input_slice=(1, 1, 2, 2, 2), weight_slice=(1, 1, 2, 2, 2), adc_bits=(6, 7, 7, 8, 8),
                     nonidealities=mf.Nonidealities(**effects))


@pytest.mark.parametrize("effects", [dict(write_variation=0.0),
                                     dict(write_variation=0.02, read_variation=0.02, voltage_variation=0.02),
                                     dict(write_variation=0.02, read_variation=0.02, read_mode="output")])
@pytest.mark.parametrize("world", [2, 3])
def test_row_shards_are_bit_identical(mf, effects, world):
    from memfast_b200.sharding import row_range, sharded_mm

    config = _config(mf, **effects)
    g = torch.Generator().manual_seed(21)
    a = torch.randn(301, 384, generator=g).cuda()
    b = torch.randn(384, 200, generator=g).cuda()
    full = mf.Simulator(config).mm(a, b)
    parts = []
    for rank in range(world):
        r0, r1 = row_range(a.shape[0], world, rank)
        parts.append(sharded_mm(a[r0:r1], b, simulator=mf.Simulator(config), row_offset=r0))
    assert torch.equal(torch.cat(parts), full)


def test_sharding_rejects_groups_across_vectors(mf):
    from memfast_b200.sharding import sharded_mm

    config = mf.Config(array_size=(128, 128), rows_per_read=32, input_quant_gran=(None, 32))
    with pytest.raises(ValueError):
        sharded_mm(torch.randn(4, 128, device="cuda"), torch.randn(128, 8, device="cuda"),
                   simulator=mf.Simulator(config), row_offset=0)
