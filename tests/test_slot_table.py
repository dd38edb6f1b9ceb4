"""Slot ownership of the persistent store (host logic, no GPU).

The scenarios are the reference's handle tests (tests/test_persistent_target_kv.py:66-98 of
qwen3-dspark): a reused slot gets a new incarnation, and a stale handle, a copy of the live
handle, an equal-valued handle built by hand and another store's handle are all refused
with ValueError; bad ids and a full table are refused with ValueError too.
"""
import copy

import pytest


def table(pkg, n):
    from importlib import import_module
    return import_module(pkg.__name__ + '.kv_store')._SlotTable(n)


def test_reuse_gives_new_incarnation_and_old_handles_die(pkg):
    t = table(pkg, 2)
    old = t.admit('same')
    assert t.index_of(old) == 0
    t.length[0] = 7
    t.release(t.index_of(old))
    fresh = t.admit('same')
    assert (fresh.index, fresh.request) == (old.index, old.request)
    assert fresh.incarnation != old.incarnation
    assert t.length[fresh.index] == 0
    for bad in (old, copy.copy(fresh), pkg.Slot(fresh.request, fresh.index, fresh.incarnation),
                table(pkg, 2).admit('same'), None, 'same', 0):
        with pytest.raises(ValueError):
            t.index_of(bad)
    assert t.index_of(fresh) == 0


def test_admission_refusals_and_lowest_free_index(pkg):
    t = table(pkg, 3)
    hs = [t.admit(r) for r in ('a', 'b', 'c')]
    assert [h.index for h in hs] == [0, 1, 2]
    for bad in ('', None, 5, 'a'):
        with pytest.raises(ValueError):
            t.admit(bad)
    with pytest.raises(ValueError):
        t.admit('d')                     # every slot taken
    t.release(t.index_of(hs[2]))
    t.release(t.index_of(hs[0]))
    assert t.admit('e').index == 0       # lowest free index first
    assert t.admit('c').index == 2       # a released id may come back
    t.length[:] = [3, 4, 5]
    assert t.resident_tokens() == 12
