"""Host logic of sequence sharding and of the attention split, on CPU: the
1M-context plan and the split count per KV group."""
import pytest

from adaptiveimi_b200 import ops, seqshard


def test_1m_context_plan_over_8_shards():
    n = 1_048_576 - 96
    plan = seqshard.plan_shards(n, 8, 2, 0.05, 32)
    assert plan.shards == 8 and sum(plan.lengths) == n
    assert plan.nprobe == 3251 and plan.max_tokens == 52424
    assert set(plan.n_slots) == {8101} and all(k == (90, 90) for k in plan.ks)
    assert plan.key_base == tuple(8101 * r for r in range(8))
    assert plan.shards * plan.cap > 8192  # the merge searches the records, not a shared-memory copy


def test_1m_context_over_2_shards_exceeds_the_slot_bound():
    # 524 K tokens per shard: k = 181, 32 762 slots > 16 384
    with pytest.raises(ValueError, match="slots per shard"):
        seqshard.plan_shards(1_048_576 - 96, 2, 2, 0.05, 32)


def test_attention_splits_per_group():
    assert ops.default_splits(8, 13200) == 18    # one CTA per SM over 8 groups
    assert ops.default_splits(4, 13200) == 37
    assert ops.default_splits(1, 13200) == 48    # capped: the split merge would cost more
    assert ops.default_splits(1, 640) == 10      # at least 64 rows per CTA
