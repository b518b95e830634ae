"""The .ignite container: the engine's writer reproduces the reference's IgniteModelWriter byte
for byte, its reader parses a container the reference wrote, and a graph saved to a container
comes back field for field (so every tensor the oracle computes is unchanged)."""
import dataclasses
import hashlib
import json

import numpy as np
import pytest

import ixb_oracle as O
from ignite_xdna_b200 import build_yolov8, random_images
from ignite_xdna_b200.container import (ARCH_XDNA1, Container, graph_from_container, graph_manifest,
                                        load_container, save_container, write_container)


def test_writer_reproduces_the_reference_writer(golden_dir, tmp_path):
    g = json.loads((golden_dir / "container_golden.json").read_text())["yolov8n_64"]
    p = tmp_path / "g.ignite"
    n = save_container(build_yolov8("n", imgsz=64), p, model_name=g["model_name"])
    assert n == g["size"]
    assert hashlib.sha256(p.read_bytes()).hexdigest() == g["sha256"]


def test_reader_parses_a_reference_written_container(golden_dir):
    with Container(golden_dir / "container_ref_small.ignite") as c:
        assert c.arch_id == ARCH_XDNA1 and c.verify()
        assert c.manifest["graph_engine"]["layers"][0]["name"] == "conv0"
        assert bytes(c.blob("engine.xclbin")) == bytes(range(200))
        assert bytes(c.blob("insts.bin")) == b"\x01\x02\x03" * 11
        assert c.blobs["wpackets.bin"]["content_type"] == "weight_packets"
        with pytest.raises(ValueError, match="NPU graph-engine"):
            graph_from_container(c)


def test_graph_round_trip(tmp_path):
    ir = build_yolov8("n", imgsz=64)
    save_container(ir, tmp_path / "m.ignite")
    ir2 = load_container(tmp_path / "m.ignite")
    assert ir2.input == ir.input and ir2.outputs == ir.outputs and ir2.task == ir.task
    assert ir2.tensors == ir.tensors
    for a, b in zip(ir.layers, ir2.layers):
        for f in dataclasses.fields(a):
            x, y = getattr(a, f.name), getattr(b, f.name)
            if isinstance(x, np.ndarray):
                assert x.dtype == y.dtype and np.array_equal(x, y), (a.name, f.name)
            elif f.name == "sigmoid" and x is not None:
                assert np.array_equal(x.table, y.table) and x.lines == y.lines and (x.s, x.ysh) == (y.s, y.ysh)
            else:
                assert x == y, (a.name, f.name)
    img = random_images(1, 64, seed=4)[0]
    r1, r2 = O.run_image(ir, img), O.run_image(ir2, img)
    assert all(np.array_equal(r1[k], r2[k]) for k in r1)


def test_reader_refuses_damaged_containers(tmp_path):
    p = tmp_path / "s.ignite"
    write_container(p, {"a": 1}, [("x", b"hello", "raw")])
    good = p.read_bytes()
    for bad, what in [(good[:-1], "declares"), (b"XXXX" + good[4:], "magic"),
                      (good[:4] + b"\x02\x00" + good[6:], "version")]:
        with pytest.raises(ValueError, match=what):
            Container(bad)
    flipped = bytearray(good)
    flipped[-64] ^= 1
    with Container(bytes(flipped)) as c:
        assert not c.verify()
