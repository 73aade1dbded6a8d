"""The card tier's books without a device (tcu_tier_new with no context, entries admitted and held through the test
hooks): the rules of src/warm.rs:62-88 (the reference's own case, warm.rs:244-271, replayed through the tier), the
hard limit on what is really on the card while evicted problems are still in use (src/gpu.rs:2560-2593), problems
larger than a tenant's budget, and concurrent use."""
import threading

from conftest import tcu


def test_ledger_rules():
    t = tcu.VramTier(None, 20, 10)
    # an entry bigger than a tenant's share is refused, and remembered as too big (never tried again)
    assert not t.debug_admit("a", "m", "p", 0, 11)
    assert t.held("a") == (0, 0)
    assert not t.debug_admit("a", "m", "p", 0, 5)
    assert t.debug_admit("a", "m", "p", 1, 6)
    # over the tenant's share: its own oldest goes
    assert t.debug_admit("b", "m", "p", 1, 6)
    assert t.debug_admit("a", "m", "p", 2, 6)
    assert t.held("a") == (12, 6) and t.debug_pin("a", "m", "p", 1) is None
    # over the overall budget: the least recently used of anyone's (b's, since a's 2 was just used)
    pin = t.debug_pin("a", "m", "p", 2)
    tcu.VramTier.debug_unpin(pin)
    assert t.debug_admit("c", "m", "p", 1, 9)
    assert t.held("a") == (15, 6) and t.debug_pin("b", "m", "p", 1) is None
    assert t.on_card("a") == (15, 6)
    assert t.ready("a") == 6 and t.ready("c") == 9
    t.evict("c", "other model")
    assert t.held("c") == (15, 9)
    t.evict("c")
    assert t.held("c") == (6, 0) and t.on_card("c") == (6, 0)
    t.evict("a")
    assert t.held("a") == (0, 0) and t.on_card("a") == (0, 0)
    # eviction forgets the too-big entry too
    assert t.debug_admit("a", "m", "p", 0, 5)
    t.free()


def test_in_use_problems_keep_their_room():
    """An evicted problem still used by a prediction stays on the card, and its bytes stay counted against the
    budgets until the prediction lets go: a new load that would not fit beside it waits (gpu.rs:2580-2586)."""
    t = tcu.VramTier(None, 10, 10)
    assert t.debug_admit("a", "m", "p", 0, 8)
    pin = t.debug_pin("a", "m", "p", 0)
    assert pin is not None
    t.evict("a")
    assert t.held("a") == (0, 0) and t.on_card("a") == (8, 8)
    assert not t.debug_admit("a", "m", "p", 1, 5)  # only 2 bytes are really free
    assert t.held("a") == (0, 0)
    assert t.debug_admit("a", "m", "p", 2, 2)
    tcu.VramTier.debug_unpin(pin)
    assert t.on_card("a") == (2, 2)
    assert t.debug_admit("a", "m", "p", 1, 5)
    assert t.on_card("a") == (7, 7)
    t.free()


def test_tenant_budget_is_at_most_the_budget():
    t = tcu.VramTier(None, 10, 100)
    assert not t.debug_admit("a", "m", "p", 0, 11)
    assert t.debug_admit("a", "m", "p", 1, 10)
    t.free()


def test_making_room_skips_entries_that_may_not_go():
    """A tenant over its share evicts only its own entries; other tenants' stay."""
    t = tcu.VramTier(None, 30, 10)
    assert t.debug_admit("a", "m", "p", 0, 10)
    assert t.debug_admit("b", "m", "p", 0, 10)
    assert t.debug_admit("a", "m", "p", 1, 4)
    assert t.held("b") == (14, 10) and t.held("a") == (14, 4)
    t.free()


def test_concurrent_admits_and_evictions_balance():
    t = tcu.VramTier(None, 1000, 400)
    stop = threading.Event()

    def tenant(name):
        for i in range(300):
            t.debug_admit(name, "m", "p", i % 7, 30 + i % 50)
            pin = t.debug_pin(name, "m", "p", (i + 3) % 7)
            all_, mine = t.on_card(name)
            assert all_ <= 1000 and mine <= 400
            if pin is not None:
                tcu.VramTier.debug_unpin(pin)

    def evictor():
        while not stop.is_set():
            t.evict("alice")

    ev = threading.Thread(target=evictor)
    ev.start()
    ths = [threading.Thread(target=tenant, args=(n,)) for n in ("alice", "bob", "carol")]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    stop.set()
    ev.join()
    for n in ("alice", "bob", "carol"):
        assert t.on_card(n)[1] == t.held(n)[1]  # nothing pinned: what is on the card is what is held
        t.evict(n)
    assert t.on_card("alice") == (0, 0) and t.held("alice") == (0, 0)
    t.free()
