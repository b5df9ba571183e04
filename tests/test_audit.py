"""Verify before fold (fault_tolerance/audit.py): a quarantined contribution
never folds until released or replaced, an attacked fleet's fold is bitwise
the honest fleet's, digests are exact and shape-aware, and the policy
replicates newcomers fully, decays veterans to a floor, bans on one
mismatch, draws its sample from the secret seed and keeps a ledger.

Would fail if an unverified gradient reached the fold, a rejected poison
changed a bit, or the policy stopped replicating newcomers, tolerated a
mismatch, or drew a sample that did not depend on the seed.
"""

import pytest
import torch

from elysium_wan_b200.fault_tolerance.audit import AuditPolicy, GatedFold, digest


def grads(seed, k=3):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(4, 5, generator=g) for _ in range(k)]


def test_quarantine_holds_every_later_index():
    f = GatedFold(range(3))
    f.add(0, grads(0))
    f.add(2, grads(2))
    f.add(1, grads(1), verified=False)
    assert f.pos == 1 and not f.complete()
    with pytest.raises(RuntimeError, match="quarantine"):
        f.result()
    f.release(1)
    assert f.complete()
    with pytest.raises(ValueError):
        f.add(0, grads(0))  # already folded


def test_rejected_poison_gives_the_honest_bits():
    honest = GatedFold(range(4))
    for mb in range(4):
        honest.add(mb, grads(mb))
    attacked = GatedFold(range(4))
    poison = [g + 1e-4 for g in grads(1)]  # below any loss-curve noise
    attacked.add(0, grads(0))
    attacked.add(1, poison, verified=False)
    attacked.add(2, grads(2))
    attacked.add(3, grads(3))
    assert digest(poison) != digest(grads(1))
    attacked.reject(1, grads(1))
    for w, g in zip(honest.result(), attacked.result()):
        assert torch.equal(w, g)
    # the fold is index order in fp32: the first assigned, the rest added
    want = [grads(0)[i].clone() for i in range(3)]
    for mb in (1, 2, 3):
        for i in range(3):
            want[i] += grads(mb)[i]
    for w, g in zip(want, honest.result()):
        assert torch.equal(w, g)


def test_released_contributions_fold_exactly():
    a, b = GatedFold(range(2)), GatedFold(range(2))
    for mb in range(2):
        a.add(mb, grads(mb))
        b.add(mb, grads(mb), verified=False)
    assert b.pos == 0
    b.release(0)
    b.release(1)
    for x, y in zip(a.result(), b.result()):
        assert torch.equal(x, y)


def test_digest_is_exact_and_shape_aware():
    assert digest(grads(7)) == digest(grads(7))
    nudged = [g.clone() for g in grads(7)]
    nudged[0][0, 0] += 2 ** -20
    assert digest(nudged) != digest(grads(7))
    assert digest([g.reshape(-1) for g in grads(7)]) != digest(grads(7))
    assert digest(grads(7)[0].to(torch.bfloat16)) != digest(grads(7)[0])


def test_newcomers_are_replicated_on_every_item():
    p = AuditPolicy(seed=b"s")
    assert all(p.replicate("new", s, m) for s in range(4) for m in range(8))


def test_veterans_decay_to_the_floor_and_stay_there():
    p = AuditPolicy(seed=b"s", warmup=4, floor=0.05, half_life=8)
    for i in range(4):
        p.record("vet", 0, i, "d", "d")
    assert p.replication_p("vet") == 1.0
    for i in range(8):
        p.record("vet", 1, i, "d", "d")
    assert p.replication_p("vet") == pytest.approx(0.5)
    for i in range(500):
        p.record("vet", 2, i, "d", "d")
    assert p.replication_p("vet") == 0.05


def test_one_mismatch_bans():
    p = AuditPolicy(seed=b"s")
    for i in range(50):
        p.record("t", 0, i, "d", "d")
    assert not p.banned("t")
    assert not p.record("t", 1, 0, "claimed", "recomputed")
    assert p.banned("t") and p.replication_p("t") == 1.0
    v = p.ledger[-1]
    assert (v.node, v.step, v.mb, v.ok) == ("t", 1, 0, False) and v.claimed != v.recomputed


def test_sortition_depends_on_the_seed_and_is_reproducible():
    a = AuditPolicy(seed=b"secret-a", warmup=0, floor=0.3, half_life=1)
    b = AuditPolicy(seed=b"secret-b", warmup=0, floor=0.3, half_life=1)
    for pol in (a, b):
        for i in range(64):
            pol.record("v", 0, i, "d", "d")
    da = [a.replicate("v", 1, m) for m in range(400)]
    db = [b.replicate("v", 1, m) for m in range(400)]
    assert da != db
    assert 0.2 < sum(da) / 400 < 0.4
    assert da == [a.replicate("v", 1, m) for m in range(400)]
    assert a.reveal() == b"secret-a"


def test_absolute_backstop_forces_an_audit():
    p = AuditPolicy(seed=b"s", warmup=0, floor=1e-9, half_life=1, absolute_every=5)
    for i in range(200):
        p.record("v", 0, i, "d", "d")
    hits = [p.replicate("v", 1, m) for m in range(50)]
    gaps, run = [], 0
    for h in hits:
        run = 0 if h else run + 1
        gaps.append(run)
    assert max(gaps) <= 4 and sum(hits) >= 10
