"""BKEX header parsing and writing of the repack module against the oracle's
restatement of kandiga/_pack_experts.py:95-132 (CPU)."""
from kandiga_b200.repack import build_header, parse_header
from oracle import oracle as O


def test_header_round_trip_matches_oracle():
    layer = O.ExpertLayer.random(4, 1024, 512, 3, seed=1, sb_dtype="bf16")
    hdr = O.bkex_header(layer.num_experts, O.bkex_tensors_for(layer))
    n, esz, tensors = parse_header(hdr)
    assert n == 3 and esz == layer.expert_size()
    assert [t["name"] for t in tensors][:3] == ["gate_proj.weight", "gate_proj.scales", "gate_proj.biases"]
    assert build_header(n, esz, tensors) == hdr
