"""The grouped launch's host-side schedule (spmm24_group_schedule, no GPU):
which K split the picker takes for the decode step and its M-shards, the
unit counts against the device's SMs and four-CTA clusters, the tuning
override, and argument checks.  The GPU side of each choice is measured
and parity-tested in tests/test_gpu_grouped.py."""
import pytest

LAYERS = ((4096, 4096), (11008, 4096), (4096, 11008))  # BASELINE config 2 (M, K); N in {1, 8, 16, 32}


def _shard(spmm24, div):
    """Rows of the first of `div` M-shards of every decode layer, four N each."""
    Ms, Ks = [], []
    for (M, K) in LAYERS:
        m = spmm24.shard_rows(M, div, 0, 128)[1]
        Ms += [m] * 4
        Ks += [K] * 4
    return Ms, Ks


@pytest.fixture
def spmm24():
    import spmm24 as s

    s.reset_tuning()
    yield s
    s.reset_tuning()


def test_decode_step_and_shards(spmm24):
    """Whole tiles for the full step (600 tiles) and a half of it; a CTA pair
    per tile for a quarter (150 tiles of 32 or 86 stages); clusters of four
    for an eighth (75 tiles), sized by the clusters that fit."""
    full = spmm24.group_schedule(*_shard(spmm24, 1))
    assert full["split"] == 1 and full["units"] == 148
    assert spmm24.group_schedule(*_shard(spmm24, 2))["split"] == 1
    quarter = spmm24.group_schedule(*_shard(spmm24, 4))
    assert quarter["split"] == 2 and quarter["units"] == 74
    eighth = spmm24.group_schedule(*_shard(spmm24, 8), max_clusters4=33)
    assert eighth["split"] == 4 and eighth["units"] == 33
    # each choice beats the others by the picker's own measure
    for gs in (1, 2):
        spmm24.set_tuning(group_split=gs)
        other = spmm24.group_schedule(*_shard(spmm24, 8), max_clusters4=33)
        assert other["split"] == gs and 10 * eighth["makespan"] < 9 * other["makespan"]
    spmm24.reset_tuning()


def test_makespan_bounds(spmm24):
    """The busiest unit carries at least the average load and at most the
    average plus the largest tile (the longest-processing-time bound)."""
    Ms, Ks = _shard(spmm24, 1)
    sc = spmm24.group_schedule(Ms, Ks)
    costs = []
    for M, K in zip(Ms, Ks):
        st = (K // 64 + 1) // 2
        costs += [st + 1] * ((M + 127) // 128)
    avg = sum(costs) / sc["units"]
    assert avg <= sc["makespan"] <= avg + max(costs)


def test_without_four_cta_clusters(spmm24):
    """No cluster of four fits (max_clusters4 = 0): never a four-way split
    unless forced, and then one cluster takes every tile."""
    sc = spmm24.group_schedule(*_shard(spmm24, 8), max_clusters4=0)
    assert sc["split"] == 2
    spmm24.set_tuning(group_split=4)
    forced = spmm24.group_schedule(*_shard(spmm24, 8), max_clusters4=0)
    assert forced["split"] == 4 and forced["units"] == 1


def test_fp8_and_small_devices(spmm24):
    """fp8 stages are 256 K (half as many); a device with few SMs gets fewer
    units, never more than the tiles."""
    Ms, Ks = _shard(spmm24, 8)
    assert spmm24.group_schedule(Ms, Ks, fp8=True)["makespan"] < spmm24.group_schedule(Ms, Ks)["makespan"]
    small = spmm24.group_schedule([128], [4096], sms=148)
    assert small["units"] == 1
    sc = spmm24.group_schedule(Ms, Ks, sms=16, max_clusters4=4)
    assert sc["units"] <= 16


@pytest.mark.parametrize("Ms,Ks,kw", [
    ([], [], {}),
    ([100], [4096], {}),            # M not a multiple of 16
    ([4096], [4000], {}),           # K not a multiple of 64
    ([4096], [4096 + 64], {"fp8": True}),  # fp8: K % 128
    ([4096], [4096], {"sms": 0}),
    ([4096], [4096], {"max_clusters4": -1}),
    ([4096] * 17, [4096] * 17, {}),  # more than 16 problems
    ([65536 * 8], [4096], {}),       # more than 2048 tiles
])
def test_bad_arguments(spmm24, Ms, Ks, kw):
    with pytest.raises(ValueError):
        spmm24.group_schedule(Ms, Ks, **kw)
