"""CPU: the ZeRO-1 partition of the training state (ne_shard_range, the
library's own host arithmetic) at 2, 4 and 8 ranks over every trainable
tensor of Qwen3-0.6B and Stories110M, listed in the order ne_train_alloc lays
them out (per layer Wqkv, Wo, W13, W2, the two norm gains and, with QK-norm,
the q/k gains; then the final norm and the embedding): every element is owned
by exactly one rank, the table every rank computes is the same, parts start
at 64-element boundaries, and the ranks' shares balance."""
import pytest

from oracle import model as om


def _segments(cfg):
    d, f, qd, kd = cfg.dim, cfg.hidden, cfg.q_dim, cfg.kv_dim
    per = [(qd + 2 * kd) * d, d * qd, 2 * f * d, d * f, d, d]
    if cfg.qk_norm:
        per += [cfg.head_dim, cfg.head_dim]
    return per * cfg.n_layers + [d, cfg.vocab * d]


@pytest.mark.parametrize("model", ["qwen3_06b", "stories110m"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_every_element_is_owned_exactly_once(model, world):
    from neural_engine_b200.runtime import shard_range
    cfg = om.PRESETS[model]
    total = [0] * world
    for n in _segments(cfg):
        # every rank computes the whole table; all of them must agree
        tables = [[shard_range(n, world, p) for p in range(world)] for _ in range(world)]
        assert all(t == tables[0] for t in tables)
        parts = tables[0]
        pos = 0
        for p, (off, ln) in enumerate(parts):
            assert off == pos and ln >= 0, (n, p, parts)
            assert off % 64 == 0, (n, p, off)
            pos += ln
            total[p] += ln
        assert pos == n, (n, parts)
    # the large tensors dominate: every rank's share within 1% of the mean
    mean = sum(total) / world
    assert max(abs(t - mean) for t in total) <= 0.01 * mean, total


def test_partition_edge_sizes():
    from neural_engine_b200.runtime import shard_range
    for n in (0, 1, 63, 64, 65, 127, 128, 1000, 4097):
        for world in (1, 2, 3, 4, 8):
            parts = [shard_range(n, world, p) for p in range(world)]
            assert sum(ln for _, ln in parts) == n
            assert [o for o, _ in parts] == sorted(o for o, _ in parts)
    with pytest.raises(Exception):
        shard_range(10, 4, 4)
