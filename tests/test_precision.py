"""Precision recipes as data (the reference's precision table, semantics
only): the boundary ladder, the representability rule behind "native",
capability gates, the e5m2 block-scale rule on the host, and the fp8 pair
codec for both formats.

Would fail if a rung went missing from the ladder, a lossy pair were called
lossless (fp16 for bf16 compute, any block-scaled fp8), the e5m2 scale
exponent drifted from 2^(e-15), or the wire lost the fp8 format.
"""

import pytest
import torch

from elysium_wan_b200 import ops
from elysium_wan_b200.models import precision
from elysium_wan_b200.models.config import make_config


def test_ladder_widest_first_and_wire_bytes():
    assert precision.LADDER == ["fp32", "bf16", "fp16", "fp8_e4m3_b128", "fp8_e5m2_b128"]
    wb = [precision.fmt(n).wire_bytes for n in precision.LADDER]
    assert wb == sorted(wb, reverse=True)
    assert precision.fmt("fp8_e5m2_b128").wire_bytes == 1 + 4 / 128


@pytest.mark.parametrize("compute,boundary,native", [
    ("bf16", "fp32", True), ("bf16", "bf16", True), ("bf16", "fp16", False),
    ("bf16", "fp8_e5m2_b128", False), ("bf16", "fp8_e4m3_b128", False),
    ("fp32", "bf16", False), ("fp32", "fp32", True), ("fp32", "fp16", False)])
def test_classification_is_representability(compute, boundary, native):
    c = precision.classify(compute, boundary)
    assert c["lossless_vs_reference"] is native
    assert c["level"] == (precision.NATIVE if native else precision.WIRE_QUANTIZED)


def test_reference_names_read_as_block_scaled():
    assert precision.fmt("fp8_e5m2").name == "fp8_e5m2_b128"
    cfg = make_config("toy", d_model=128, n_head=4, boundary_dtype="fp8_e4m3")
    assert cfg.boundary_dtype == "fp8_e4m3_b128" and cfg.fp8_boundary()
    with pytest.raises(ValueError):
        precision.fmt("fp4")


def test_compute_capability_gates():
    assert precision.compute_runnable("bf16", (10, 0))
    assert not precision.compute_runnable("bf16", (9, 0))
    assert precision.compute_runnable("bf16", None)
    assert precision.compute_runnable("fp32", (7, 0))
    assert not precision.compute_runnable("fp16", (10, 0))  # not built


def test_describe_prices_the_wire():
    d = precision.describe("bf16", "fp8_e5m2_b128", 5120, wire_ratio=1.25)
    assert d["wire_bytes_per_token_raw"] == 5120 * (1 + 4 / 128)
    assert d["needs_scale"] and not d["lossless_vs_reference"]


def test_host_e5m2_block_scale_rule():
    torch.manual_seed(0)
    x = torch.randn(16, 512) * torch.logspace(-6, 6, 16)[:, None]
    q, s = ops.quant_q8(x, ops.E5M2)
    amax = x.view(16, 4, 128).abs().amax(-1)
    e = torch.frexp(amax)[1]
    assert torch.equal(s, torch.ldexp(torch.ones_like(amax), e - 15))
    back = ops.dequant_q8(q, s, torch.float32)
    assert ((back - x).abs() <= x.abs() * 2.0 ** -3 + s.repeat_interleave(128, 1) * 2.0 ** -16).all()


@pytest.mark.parametrize("dt", [ops.E4M3, ops.E5M2])
def test_fp8_pair_codec_keeps_the_format(dt):
    from elysium_wan_b200.transport import framing

    q, s = ops.quant_q8(torch.randn(8, 256), dt)
    cid, payload, shape = framing.encode_tensor((q, s), "planes")
    f = framing.Frame(type=framing.FWD, codec=cid, step=0, mb=0, chunk=0, payload=payload,
                      shape=shape)
    q2, s2 = f.tensor()
    assert q2.dtype == dt
    assert torch.equal(q2.view(torch.uint8), q.view(torch.uint8)) and torch.equal(s2, s)


def test_admission_ladder_prices_every_rung():
    from elysium_wan_b200.scheduler import autoconfig

    cfg = make_config("gpt15b", n_layer=4)
    rows = autoconfig.evaluate(cfg, params_stage=10**9, n_layers_stage=4, mb_size=1,
                               live_graphs=2, link_mbps=1000.0, window_s=1.0,
                               mem_budget_bytes=170e9)
    assert [r["boundary"] for r in rows] == precision.LADDER
    by = {r["boundary"]: r for r in rows}
    assert by["bf16"]["lossless"] and not by["fp16"]["lossless"]
    assert by["fp8_e5m2_b128"]["needs_scale"] and not by["fp16"]["needs_scale"]
    assert by["fp16"]["floor_mbps"] == by["bf16"]["floor_mbps"]
