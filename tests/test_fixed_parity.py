"""Bit-exact parity of the fixed-page metadata runtime (Fixed-8/16/32/64)
against the reference's own FixedPageManager compiled from its sources.

Identical seeded operation streams (create / append / reserve / commit /
rollback / seal / fork / release, valid and invalid) run on the product
(kkrt_fixed_*) and on the reference (kref_fixed_*). Every return value,
reservation table, block table, snapshot and invariant verdict must match.
Small pools make exhaustion and staged-page rollback frequent.
"""
import random

import pytest


class FixedPair:
    def __init__(self, kk, kk_lib, ref_lib, tokens, capacity):
        self.a = kk.FixedManager(kk_lib, "kkrt_", tokens, capacity)
        self.b = kk.FixedManager(ref_lib, "kref_", tokens, capacity)
        self.tokens = tokens

    def same(self, name, *args):
        ra = getattr(self.a, name)(*args)
        rb = getattr(self.b, name)(*args)
        assert ra == rb, f"{name}{args}: product={ra} reference={rb}"
        return ra

    def full_check(self, ids):
        assert self.a.snapshot() == self.b.snapshot()
        for rid in ids:
            self.same("table", rid)
        assert self.a.invariants() and self.b.invariants()


def run_fixed_stream(pair: FixedPair, seed: int, steps: int):
    rng = random.Random(seed)
    ids = list(range(1, 11))
    reservations = []
    T = pair.tokens
    for step in range(steps):
        op = rng.random()
        rid = rng.choice(ids + [0])
        if op < 0.10:
            pair.same("create", rid)
        elif op < 0.30:
            pair.same("append", rid, rng.choice([0, 1, 2, T - 1, T, T + 1, 2 * T + 3, 5 * T, 100]))
        elif op < 0.50:
            t = pair.a.table(rid)
            count = sum(e[1] for e in t[1]) if t else 0
            expected = count if rng.random() < 0.85 else count + rng.choice([-1, 1])
            err, res_id, _, _ = pair.same("reserve", rid, max(expected, 0))
            if err == 0:
                reservations.append(res_id)
        elif op < 0.65 and reservations:
            res_id = reservations.pop(rng.randrange(len(reservations)))
            pair.same("commit" if rng.random() < 0.7 else "rollback", res_id)
        elif op < 0.70:
            pair.same("commit" if rng.random() < 0.5 else "rollback", rng.randrange(0, 4))
        elif op < 0.78:
            pair.same("seal", rid)
        elif op < 0.88:
            pair.same("fork", rid, rng.choice(ids + [0]))
        else:
            pair.same("release", rid)
        if step % 7 == 0:
            pair.full_check(ids)
    pair.full_check(ids)


@pytest.mark.parametrize("tokens", [8, 16, 32, 64, 1, 5])
@pytest.mark.parametrize("seed", range(3))
def test_fixed_streams_match_reference(kk, kk_lib, ref_lib, tokens, seed):
    capacity = [12, 40, 3][seed % 3]
    run_fixed_stream(FixedPair(kk, kk_lib, ref_lib, tokens, capacity), seed * 31 + tokens, 700)


def test_fixed_decode_with_fork_and_partial_tail_cow(kk, kk_lib, ref_lib):
    """A decode-shaped sequence: prefill appends, forks at partial tails,
    then one reserved token per request per step, committed."""
    for tokens in (8, 16, 32, 64):
        pair = FixedPair(kk, kk_lib, ref_lib, tokens, 512)
        for rid, ctx in [(1, 17), (2, 100), (3, 513), (4, 64)]:
            assert pair.same("create", rid) == 0
            assert pair.same("append", rid, ctx) == 0
        assert pair.same("fork", 3, 9) == 0
        assert pair.same("fork", 1, 10) == 0
        for _ in range(70):
            for rid in (1, 2, 3, 4, 9, 10):
                count = sum(e[1] for e in pair.a.table(rid)[1])
                err, res_id, _, reserved = pair.same("reserve", rid, count)
                assert err == 0
                assert pair.same("commit", res_id) == 0
        pair.full_check([1, 2, 3, 4, 9, 10])
        for rid in (1, 2, 3, 4, 9, 10):
            assert pair.same("release", rid) == 0
        assert pair.a.snapshot()[4][2] == 0   # pool: nothing allocated


def test_fixed_rejects_zero_sizes(kk, kk_lib, ref_lib):
    for lib, prefix in ((kk_lib, "kkrt_"), (ref_lib, "kref_")):
        with pytest.raises(ValueError):
            kk.FixedManager(lib, prefix, 0, 8)
        with pytest.raises(ValueError):
            kk.FixedManager(lib, prefix, 8, 0)
        m = kk.FixedManager(lib, prefix, 16, 4)
        assert m.tokens_per_page() == 16
