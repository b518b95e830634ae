"""The CPU oracle against the reference's own outputs (fixtures from tests/golden/make_golden.py)."""
import hashlib
import json

import numpy as np
import pytest

import ixb_oracle as O
from ignite_xdna_b200 import build_yolov8, random_images
from ignite_xdna_b200 import silu


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def kat(golden_dir):
    return np.load(golden_dir / "kat.npz")


@pytest.fixture(scope="module")
def hashes(golden_dir):
    return json.loads((golden_dir / "graph_hashes.json").read_text())


def test_rne_shift_matches_reference(kat):
    x = np.arange(-70000, 70000, dtype=np.int64)
    for s in (0, 1, 2, 5, 9, 12, 16):
        assert np.array_equal(O.rne_shift(x, s), kat[f"rne_{s}"]), s
        assert np.array_equal(silu.rne_shift(x, s), kat[f"rne_{s}"]), s


def test_rne_shift_is_bankers_rounding():
    """The reference's own check (tests/test_conv_engine.py:363-367)."""
    x = np.arange(-4096, 4096, dtype=np.int64)
    for s in (1, 2, 5, 9):
        assert np.array_equal(O.rne_shift(x, s), np.round(x / (1 << s)).astype(np.int64))


def test_float_shift_round_saturate_equals_the_integer_rule():
    """The conv epilogue computes sat_s8(rne(c / 2^s)) as float32(c) (round to nearest) times 2^-s,
    converted back rounding half to even with saturation. The same float32 steps here must equal
    clip(rne_shift(c, s)) for every shift the engine accepts, across the whole int32 range (exact:
    float32 holds every |c| < 2^24, and larger values saturate either way)."""
    c = np.concatenate([np.arange(-70000, 70000), np.array([-2 ** 31, 2 ** 31 - 1, 2 ** 24 - 1, 2 ** 24 + 1,
                                                           -(2 ** 24) - 3, 127 << 16, (127 << 16) + (1 << 15)]),
                        np.random.default_rng(5).integers(-2 ** 31, 2 ** 31, 300000)]).astype(np.int64)
    for s in range(17):
        f = c.astype(np.float32) * np.float32(2.0 ** -s)
        got = np.clip(np.rint(f), -128, 127).astype(np.int64)   # rint: round half to even
        assert np.array_equal(got, np.clip(O.rne_shift(c, s), -128, 127)), s


def test_residual_rule_matches_reference(kat):
    tm, tr = np.meshgrid(np.arange(256), np.arange(256), indexing="ij")
    keys = [k for k in kat.files if k.startswith("res_")]
    assert len(keys) >= 6
    for key in keys:
        a, b, s = (int(v) for v in key.split("_")[1:])
        got = O.residual_combine(tm.astype(np.uint8), tr.astype(np.uint8), s, a, b)
        assert np.array_equal(got, kat[key]), key


def test_residual_rule_is_float_add():
    """Exhaustive check against the float Add (tests/test_graph_engine_offline.py:310-323)."""
    tm, tr = np.meshgrid(np.arange(256), np.arange(256), indexing="ij")
    for s_main, s_res, s_out in ((0.03125, 0.0625, 0.0625), (0.125, 0.0625, 0.0625), (4.0, 2.0, 4.0)):
        s_min = min(s_main, s_res)
        a, b, sh = (int(round(np.log2(v / s_min))) for v in (s_main, s_res, s_out))
        got = O.residual_combine(tm.astype(np.uint8), tr.astype(np.uint8), sh, a, b)
        x = (tm - 128) * s_main + (tr - 128) * s_res
        ref = np.clip(np.round(x / s_out) + 128, 0, 255).astype(np.uint8)
        assert np.array_equal(got, ref)


def test_sigmoid_tables_match_reference(kat):
    pairs = kat["sig_pairs"]
    assert len(pairs) >= 5
    for s1, s2 in pairs:
        fit = silu.fit_sigmoid(float(s1), float(s2))
        key = f"sig_{float(s1)!r}_{float(s2)!r}"
        assert np.array_equal(fit.table, kat[key + "_table"]), key
        assert np.array_equal(np.array(fit.lines), kat[key + "_lines"]), key
        assert [fit.s, fit.ysh] == list(kat[key + "_s_ysh"]), key


def test_int4_packing_matches_reference(kat):
    assert np.array_equal(O.pack_int4(np.arange(-8, 8)), kat["int4_pack_range"])
    assert O.pack_int4(np.array([3, -5]))[0] == 0xB3 == kat["int4_pack_3_m5"][0]
    assert np.array_equal(O.pack_int4(kat["int4_b"]), kat["int4_b_packed"])
    assert np.array_equal(O.unpack_int4(kat["int4_b_packed"]), kat["int4_b"])


@pytest.mark.parametrize("imgsz,task", [(64, "detect"), (96, "detect"), (64, "pose")])
def test_small_graph_every_tensor(golden_dir, imgsz, task):
    """YOLOv8-pose adds one-class heads and 51-channel keypoint branches (channels that are not
    whole 16-channel chunks)."""
    tag = "_pose" if task == "pose" else ""
    z = np.load(golden_dir / f"yolov8n{tag}_s{imgsz}.npz")
    ir = build_yolov8("n", imgsz=imgsz, task=task)
    for i, im in enumerate(z["images"]):
        t = O.run_image(ir, im)
        names = [k.split("|", 1)[1] for k in z.files if k.startswith(f"{i}|")]
        assert len(names) == len(ir.layers) + 1
        for n in names:
            assert np.array_equal(t[n], z[f"{i}|{n}"]), n


@pytest.mark.parametrize("variant", ["n", "s", "m"])
def test_full_graph_hashes(hashes, variant):
    ir = build_yolov8(variant, imgsz=640)
    h = hashes[f"yolov8{variant}"]
    t = O.run_image(ir, random_images(1, 640, seed=h["image_seed"])[0])
    bad = [n for n, v in h["tensors"].items() if sha(t[n]) != v]
    assert not bad, bad[:5]
    heads = O.heads_int8(ir, t)
    for name, v in h["heads"].items():
        assert sha(heads[name][0]) == v, name


def test_pose_graph_hashes(golden_dir):
    h = json.loads((golden_dir / "pose_hashes.json").read_text())["yolov8n-pose"]
    ir = build_yolov8("n", imgsz=640, task="pose")
    assert sorted(h["heads"]) == sorted(n for n, _ in ir.outputs)
    t = O.run_image(ir, random_images(1, 640, seed=h["image_seed"])[0])
    bad = [n for n, v in h["tensors"].items() if sha(t[n]) != v]
    assert not bad, bad[:5]
    heads = O.heads_int8(ir, t)
    assert [heads[n].shape[1] for n in ("p3_cls", "p3_kpt")] == [1, 51]
    for name, v in h["heads"].items():
        assert sha(heads[name][0]) == v, name


def test_u8i4_oracle_matches_reference_known_answers(golden_dir):
    kat = np.load(golden_dir / "u8i4_kat.npz")
    for i in range(6):
        assert np.array_equal(O.u8i4_i32(kat[f"a{i}"], kat[f"b{i}_packed"]), kat[f"c{i}"])
