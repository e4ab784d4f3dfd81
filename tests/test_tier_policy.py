"""The expert cache's replacement policies (oomb_policy, host-only): the cases of
the reference's own policy tests (crates/oominf-tiers/src/policy.rs:140-169)."""
import pytest

from homelab_b200.stage import Policy


def test_lru_evicts_oldest_unpinned():
    p = Policy("lru")
    for t, k in enumerate([1, 2, 3]):
        p.touch(k, t)
    p.touch(1, 10)
    assert p.victim() == 2
    assert p.victim([2]) == 3
    p.remove(2)
    assert p.victim() == 3


def test_lrfu_prefers_frequent_and_decays():
    p = Policy("lrfu:1e9")  # effectively LFU
    p.touch(1, 0)
    p.touch(1, 1)
    p.touch(2, 2)
    assert p.victim() == 2
    q = Policy("lrfu:1.0")  # strong decay: recency wins
    q.touch(1, 0)
    q.touch(1, 1)
    q.touch(2, 10)
    assert q.victim() == 1


def test_lfu_and_empty_and_all_pinned():
    p = Policy("lfu")
    assert p.victim() is None
    p.touch(5, 0)
    p.touch(5, 1)
    p.touch(6, 2)
    assert p.victim() == 6
    assert p.victim([5, 6]) is None


@pytest.mark.parametrize("spec", ["mru", "lrfu:", "lrfu:x", "lrfu:-1"])
def test_unknown_policies_are_refused(spec):
    from homelab_b200._lib import OombError
    with pytest.raises(OombError):
        Policy(spec)
