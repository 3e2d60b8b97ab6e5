"""Host logic of Lax.psumSgdTree's fused path (no GPU): the bucket plan, the
peer-buffer layout, and which trees take the fused path."""
from jax4j_b200 import psum_sgd as PS


def test_buckets_walk_from_the_last_leaf_and_close_on_size_or_segments():
    sizes = [196608, 384, 99840, 260] + [4 * (k + 1) for k in range(18)] + [307200]
    b = PS.plan_buckets(sizes, 262144)
    assert b[0] == [22]                       # the last leaf alone reaches the bucket size
    assert b[1] == list(range(21, 5, -1))     # 16 leaves: the segment limit
    assert b[2] == [5, 4, 3, 2, 1, 0]
    assert sorted(i for x in b for i in x) == list(range(len(sizes)))


def test_layout_keeps_every_area_16_byte_aligned():
    sizes = [1000, 4096 * 1000, 4096, 1024 * 4096]
    buckets = PS.plan_buckets(sizes, 1 << 22)
    g, u, total = PS.layout(sizes, buckets)
    lens = [sum(sizes[i] for i in bb) for bb in buckets]
    assert g[0] == PS.FLAG_AREA
    for off in g + u:
        assert off % 16 == 0
    assert u[0] == g[-1] + 4 * lens[-1]
    assert total == u[-1] + 4 * lens[-1]
