"""Bit-exact parity of the page-metadata runtime against the reference.

Identical seeded operation streams (create / append / reserve / commit /
rollback / seal / fork / release / promotion prepare-commit-rollback / leases,
valid and invalid) run on the product KvCacheManager (kkrt_*) and on the
reference's own KvCacheManager compiled from its sources (kref_*). Every
return value, reservation table, promotion handle set, lease, block table,
page metadata record, pool snapshot and invariant verdict must be identical.
Small pools make exhaustion and rollback paths frequent.
"""
import random

import pytest


class Pair:
    def __init__(self, kk, kk_lib, ref_lib, micro, extent):
        self.a = kk.Manager(kk_lib, "kkrt_", micro, extent)
        self.b = kk.Manager(ref_lib, "kref_", micro, extent)
        self.handles = set()

    def same(self, name, *args):
        ra = getattr(self.a, name)(*args)
        rb = getattr(self.b, name)(*args)
        assert ra == rb, f"{name}{args}: product={ra} reference={rb}"
        self._collect(ra)
        return ra

    def _collect(self, value):
        # remember every page handle ever reported so stale ones get queried too
        if isinstance(value, tuple):
            if len(value) == 5 and all(isinstance(v, int) for v in value):
                begin, valid, kind, slot, gen = value
                self.handles.add((kind, slot, gen))
            elif len(value) == 3 and all(isinstance(v, int) for v in value) and value[2] > 0:
                self.handles.add(value)
            for v in value:
                self._collect(v)

    def full_check(self, request_ids):
        assert self.a.snapshot() == self.b.snapshot()
        for rid in request_ids:
            self.same("table", rid)
        for h in sorted(self.handles):
            self.same("page_meta", *h)
        ia, ib = self.a.invariants(), self.b.invariants()
        assert ia == ib
        assert ia, "invariants must hold after every operation"


def run_stream(pair: Pair, seed: int, steps: int):
    rng = random.Random(seed)
    ids = list(range(1, 13))
    tokens = {}          # request -> committed token count (as seen through results)
    reservations = []    # (reservation id, request id)
    promotions = []
    leases = []
    for step in range(steps):
        op = rng.random()
        rid = rng.choice(ids + [0])
        if op < 0.08:
            pair.same("create", rid)
        elif op < 0.22:
            pair.same("append", rid, rng.choice([0, 1, 2, 3, 5, 7, 8, 9, 15, 16, 17, 40, 64, 70]))
        elif op < 0.40:
            t = pair.a.table(rid)
            count = sum(e[1] for e in t[1]) if t else 0
            expected = count if rng.random() < 0.85 else count + rng.choice([-1, 1])
            err, res_id, before, reserved = pair.same("reserve", rid, max(expected, 0))
            if err == 0:
                reservations.append(res_id)
        elif op < 0.52 and reservations:
            res_id = reservations.pop(rng.randrange(len(reservations)))
            if rng.random() < 0.3:
                err, lid, n = pair.same("lease_reservation", res_id)
                if err == 0:
                    leases.append(lid)
            pair.same("commit" if rng.random() < 0.7 else "rollback", res_id)
        elif op < 0.57:
            pair.same("seal", rid)
        elif op < 0.64:
            pair.same("fork", rid, rng.choice(ids + [0]))
        elif op < 0.70:
            pair.same("release", rid)
        elif op < 0.80:
            t = pair.a.table(rid)
            begins = [e[0] for e in t[1]] if t else [0]
            begin = rng.choice(begins + [3])
            err, pid, src, tgt = pair.same("prepare_promotion", rid, begin)
            if err == 0:
                promotions.append(pid)
        elif op < 0.88 and promotions:
            pid = rng.choice(promotions)
            r = rng.random()
            if r < 0.25:
                err, lid, n = pair.same("lease_promotion", pid)
                if err == 0:
                    leases.append(lid)
            elif r < 0.7:
                if pair.same("commit_promotion", pid) in (0, 9, 10, 11):
                    promotions.remove(pid)
            else:
                pair.same("rollback_promotion", pid)
                promotions.remove(pid)
        elif op < 0.94:
            err, lid, n = pair.same("lease_request", rid)
            if err == 0:
                leases.append(lid)
        elif leases:
            lid = leases.pop(rng.randrange(len(leases)))
            pair.same("release_lease", lid)
        else:
            pair.same("release_lease", rng.randrange(0, 5))
        if step % 7 == 0:
            pair.full_check(ids)
    pair.full_check(ids)


@pytest.mark.parametrize("seed", range(12))
def test_random_op_streams_match_reference(kk, kk_lib, ref_lib, seed):
    micro, extent = [(48, 6), (24, 2), (200, 16), (9, 1)][seed % 4]
    pair = Pair(kk, kk_lib, ref_lib, micro, extent)
    run_stream(pair, seed, 900)


def run_promotion_stream(pair: Pair, seed: int, steps: int):
    """Promotion-heavy mix: long appends, several promotions pending on one
    request at once, promotion IO leases, reads leases that retire pages, and
    releases of requests that still have pending promotions (their rollback
    order is observable through the free list)."""
    rng = random.Random(1000 + seed)
    ids = list(range(1, 7))
    pending = []
    leases = []
    for step in range(steps):
        rid = rng.choice(ids)
        op = rng.random()
        if op < 0.10:
            pair.same("create", rid)
        elif op < 0.25:
            pair.same("append", rid, rng.choice([8, 16, 64, 70, 128, 131, 200]))
        elif op < 0.30:
            pair.same("seal", rid)
        elif op < 0.55:
            t = pair.a.table(rid)
            if not t:
                continue
            micro_begins = [e[0] for e in t[1] if e[2] == 0]
            if not micro_begins:
                continue
            err, pid, _, _ = pair.same("prepare_promotion", rid, rng.choice(micro_begins))
            if err == 0:
                pending.append(pid)
        elif op < 0.70 and pending:
            pid = rng.choice(pending)
            r = rng.random()
            if r < 0.3:
                err, lid, _ = pair.same("lease_promotion", pid)
                if err == 0:
                    leases.append(lid)
            elif r < 0.8:
                pair.same("commit_promotion", pid)
                pending.remove(pid)
            else:
                pair.same("rollback_promotion", pid)
                pending.remove(pid)
        elif op < 0.78:
            err, lid, _ = pair.same("lease_request", rid)
            if err == 0:
                leases.append(lid)
        elif op < 0.86 and leases:
            pair.same("release_lease", leases.pop(rng.randrange(len(leases))))
        elif op < 0.93:
            pair.same("release", rid)
        else:
            pair.same("fork", rid, rng.choice(ids))
        if step % 5 == 0:
            pair.full_check(ids)
    pair.full_check(ids)


@pytest.mark.parametrize("seed", range(6))
def test_promotion_heavy_streams_match_reference(kk, kk_lib, ref_lib, seed):
    pair = Pair(kk, kk_lib, ref_lib, 400, [4, 12, 40][seed % 3])
    run_promotion_stream(pair, seed, 700)


def test_prefill_promote_decode_sequence(kk, kk_lib, ref_lib):
    """The config-1/config-4 table build: append a body, seal, promote every
    aligned 64-token run, then decode one token at a time with forks."""
    prefill_promote_decode(Pair(kk, kk_lib, ref_lib, 4096, 128))


def prefill_promote_decode(pair: Pair):
    for rid, ctx in [(1, 17), (2, 100), (3, 513), (4, 2000)]:
        pair.same("create", rid)
        pair.same("append", rid, ctx)
        pair.same("seal", rid)
        for begin in range(0, (ctx // 64) * 64, 64):
            err, pid, _, _ = pair.same("prepare_promotion", rid, begin)
            assert err == 0
            err, lid, n = pair.same("lease_promotion", pid)
            assert err == 0 and n == 9
            assert pair.same("release_lease", lid) == 0
            assert pair.same("commit_promotion", pid) == 0
    pair.same("fork", 3, 9)
    for step in range(20):
        for rid in (1, 2, 3, 4, 9):
            t = pair.a.table(rid)
            count = sum(e[1] for e in t[1])
            err, res_id, _, reserved = pair.same("reserve", rid, count)
            assert err == 0
            err, lid, _ = pair.same("lease_reservation", res_id)
            assert err == 0
            assert pair.same("release_lease", lid) == 0
            assert pair.same("commit", res_id) == 0
    pair.full_check([1, 2, 3, 4, 9])
