"""DS41PK01 pack writer/reader on the CPU: header and index fields in the reference's slot layout
(runtime/ds41/cache.py:40-43, tools/pack_exl3.py:77-112,188-199), byte-exact records, expert subsets."""
import struct

import numpy as np
import pytest
import torch

from eva_b200 import config as C
from eva_b200.experts import make_layer, record_layout
from eva_b200.pack import MUL1_MULT, Pack, load_layer, write_pack

SMALL = C.MoEConfig("small", hidden=256, inter=128, n_experts=6, topk=2, router="softmax", shared_inter=256, bits=3,
                    shared_bits=4)
# the reference reader's slot struct, written out independently of eva_b200.pack
REF_SLOT = struct.Struct("<QIHH" + "HHHHIIIiIII" * 3)


@pytest.fixture
def packed(tmp_path):
    layers = [make_layer(SMALL, "cpu", seed=s) for s in (1, 2)]
    path = tmp_path / "experts.bin"
    write_pack(str(path), layers)
    return path, layers


def test_header_and_index_follow_the_reference_layout(packed):
    path, layers = packed
    raw = path.read_bytes()
    assert raw[:8] == b"DS41PK01"
    version, n_layers, n_experts, slot = struct.unpack("<IIII", raw[8:24])
    assert (version, n_layers, n_experts, slot) == (1, 2, 6, 128)
    offs, padded, shapes = record_layout(SMALL.hidden, SMALL.inter, SMALL.bits)
    seen = set()
    for i in range(n_layers * n_experts):
        f = REF_SLOT.unpack_from(raw, 24 + i * 128)
        rec_off, nbytes, k0, one = f[:4]
        assert nbytes == padded and k0 == 3 and one == 1 and rec_off % 4096 == 0
        seen.add(rec_off)
        for pi, proj in enumerate(("gate", "down", "up")):
            in_f, out_f, k, pad, suh_b, svh_b, tr_b, mul1, r_suh, r_svh, r_tr = f[4 + 11 * pi: 15 + 11 * pi]
            assert (in_f, out_f) == shapes[proj] and k == 3 and pad == 0
            assert suh_b == in_f * 2 and svh_b == out_f * 2 and tr_b == in_f * out_f * 3 // 8
            assert mul1 & 0xFFFFFFFF == MUL1_MULT
            assert (r_suh, r_svh, r_tr) == (offs[(proj, "suh")][0], offs[(proj, "svh")][0], offs[(proj, "trellis")][0])
            assert r_svh == r_suh + suh_b and r_tr == r_svh + svh_b
    assert len(seen) == n_layers * n_experts
    assert len(raw) == max(seen) + padded


def test_records_round_trip_byte_exact(packed):
    path, layers = packed
    pack = Pack.open(str(path))
    rec = layers[0].record_bytes
    for li, lay in enumerate(layers):
        back = load_layer(pack, li, lay)
        assert torch.equal(back.storage, lay.storage)
        assert torch.equal(back.packed - back.storage.data_ptr(), lay.packed - lay.storage.data_ptr())
        for e in range(SMALL.n_experts):
            assert pack.record(li, e) == lay.storage[e * rec:(e + 1) * rec].numpy().tobytes()


def test_expert_subset_and_shape_checks(packed, tmp_path):
    path, layers = packed
    pack = Pack.open(str(path))
    sub = load_layer(pack, 1, layers[1], experts=(5, 0, 3))
    full = make_layer(SMALL, "cpu", seed=2, experts=(5, 0, 3))
    assert torch.equal(sub.storage, full.storage) and sub.experts == (5, 0, 3)
    with pytest.raises(ValueError):
        load_layer(pack, 0, make_layer(SMALL.with_(bits=4), "cpu", seed=1))
    bad = tmp_path / "bad.bin"
    bad.write_bytes(b"NOTAPACK" + bytes(64))
    with pytest.raises(ValueError):
        Pack.open(str(bad))


def test_pack_matches_the_reference_packer(tmp_path):
    """The reference's own tools/pack_exl3.py, run on the same seeded experts (make_pack_pin.py),
    wrote the same header, the same index fields apart from the record offset, and the same record
    bytes as write_pack."""
    import hashlib
    import json
    from pathlib import Path
    pin = json.loads((Path(__file__).resolve().parent / "golden" / "pack_ref_pin.json").read_text())
    cfg = C.MoEConfig(**pin["config"])
    layers = [make_layer(cfg, "cpu", seed=s) for s in pin["seeds"]]
    path = tmp_path / "experts.bin"
    write_pack(str(path), layers)
    raw = path.read_bytes()
    assert raw[:8].decode() == pin["magic"]
    assert list(struct.unpack("<IIII", raw[8:24])) == pin["header"]
    pack = Pack.open(str(path))
    for i, (ref_slot, ref_sha) in enumerate(zip(pin["slots"], pin["record_sha256"])):
        ours = pack.slots[i]
        assert list(ours[1:]) == ref_slot[1:]
        assert hashlib.sha256(raw[ours[0]: ours[0] + ours[1]]).hexdigest() == ref_sha
