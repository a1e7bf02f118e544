"""CPU tests of the DiT block module's host logic: the attention's head-group count follows Dit::attn_groups
(dit.rs:762-773)."""
from h3q import dit as D


def test_attn_groups_follows_the_reference_rule():
    # 3 * tokens * hidden * 2 bytes of bf16 qkv against the 1.5e9-byte budget, then the next divisor of heads
    assert D.attn_groups(32760, 40, 5120) == 1                 # 1.006e9 bytes: one group
    assert D.attn_groups(65520, 40, 5120) == 2                 # 2.01e9: two budgets, 40 % 2 == 0
    assert D.attn_groups(120000, 40, 5120) == 4                # 3.69e9: three budgets, next divisor of 40 is 4
    assert D.attn_groups(200000, 40, 5120) == 5                # 6.14e9: five budgets
    assert D.attn_groups(10 ** 7, 40, 5120) == 40              # more budgets than heads: one head per group
    assert D.attn_groups(32760, 40, 5120, override=8) == 8     # H3_ATTN_GROUPS, a divisor of heads
    assert D.attn_groups(10 ** 7, 40, 5120, override=3) == 1   # not a divisor: one group
    assert D.attn_groups(10 ** 7, 40, 5120, override=0) == 1
