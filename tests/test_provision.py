"""Data provisioning: a data-reading slot fetches and verifies exactly the
shards its microbatches draw; corrupt bytes are re-fetched; without a source
it refuses by name; a manifest other than the planned one is refused."""

import os

import pytest

from elysium_wan_b200.models import dataset as ds
from elysium_wan_b200.models import provision as pv
from elysium_wan_b200.models.config import make_config
from elysium_wan_b200.runtime.spec import JobSpec


def _corpus(d, shards=4):
    txt = os.path.join(d, "corpus.txt")
    with open(txt, "w") as f:
        for i in range(200):
            f.write(f"line {i} of a small corpus for provisioning tests\n")
    out = os.path.join(d, "tokens.bin")
    ds.prepare(txt, out, tokenizer="bytes", source_type="text", n_shards=shards)
    return out


def test_slot_fetches_its_shards_and_refetches_corruption(tmp_path):
    src = tmp_path / "src"
    dst = tmp_path / "node"
    src.mkdir()
    dst.mkdir()
    made = _corpus(str(src))
    spec = JobSpec(model=make_config("toy", vocab_size=256), stages=2, stage_widths=[2, 1],
                   microbatches=4, mb_size=1, data_shards=4,
                   dataset_path=str(dst / "tokens.bin"), dataset_source=str(src),
                   dataset_sha256=pv.manifest_digest(made)).finalize()
    # peer 0 of stage 0 owns microbatches 0 and 2 -> shards {0, 2}
    assert pv.needed_shards(spec, 0, 0) == sorted({mb % 4 for mb in spec.owned(0, 0)})
    assert pv.needed_shards(spec, 1, 0) == [0, 1, 2, 3]
    rep = pv.provision_slot(spec, 0, 0)
    assert sorted(rep["fetched"]) == pv.needed_shards(spec, 0, 0)
    # a second call verifies from the stamps and fetches nothing
    assert pv.provision_slot(spec, 0, 0)["fetched"] == []
    k = pv.needed_shards(spec, 0, 0)[0]
    shard = dst / f"tokens.bin.shard{k}of4"
    b = bytearray(shard.read_bytes())
    b[0] ^= 0xFF
    shard.write_bytes(bytes(b))
    assert k in pv.provision_slot(spec, 0, 0)["fetched"]


def test_refusals(tmp_path):
    src = tmp_path / "src"
    src.mkdir()
    made = _corpus(str(src))
    nodir = tmp_path / "empty"
    nodir.mkdir()
    with pytest.raises(pv.DataRefused):
        pv.provision(str(nodir / "tokens.bin"), [0], 4)  # nothing local, no source
    with pytest.raises(pv.DataRefused):
        pv.ensure_manifest(made, pinned="0" * 64)  # another corpus than planned
    # a middle stage reads nothing
    spec = JobSpec(model=make_config("toy", vocab_size=256), stages=3, microbatches=2, mb_size=1,
                   dataset_path=made).finalize()
    assert pv.provision_slot(spec, 1, 0) is None
