"""Generate the golden fixtures by running the reference's own integer reference.

Run with ``IXB_REFERENCE`` set to the reference checkout's root:
``IXB_REFERENCE=<checkout> python tests/golden/make_golden.py``.

The reference's ``src/ignite_xdna/__init__.py`` and ``compiler/__init__.py`` import
onnx-dependent modules eagerly and onnx is not installed, so the four modules this path
needs (``engine_emulator``, ``silu_sigmoid``, ``graph_ir``, ``graph_reference``) are loaded
by file path under empty stand-in packages. Nothing else of the reference is executed.

Outputs (all small, committed):
* ``kat.npz``            known answers: rne_shift, residual rule, sigmoid tables, int4 packing
* ``yolov8n_s64.npz``    every tensor of run_direct on a 64x64 YOLOv8n, two images
* ``yolov8n_s96.npz``    the same at 96x96
* ``graph_hashes.json``  per-tensor sha256 of run_direct at 640x640 for YOLOv8n/s/m (one image
                         each) plus a fingerprint of each synthetic model
* ``yolov8n_pose_s64.npz`` every tensor of run_direct on a 64x64 YOLOv8n-pose, two images, and
  ``pose_hashes.json`` its per-tensor sha256 at 640x640 (``--pose`` writes only these two)
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("IXB_REFERENCE", ""))


def require_reference() -> None:
    """The generators read the reference's own sources: IXB_REFERENCE must name its checkout."""
    if not os.environ.get("IXB_REFERENCE") or not (REF / "src" / "ignite_xdna").is_dir():
        raise SystemExit("set IXB_REFERENCE to the reference checkout's root (the tree holding src/ignite_xdna)")
sys.path.insert(0, str(REPO))

from ignite_xdna_b200 import build_yolov8, random_images  # noqa: E402
from ignite_xdna_b200.graph import ConvLayer  # noqa: E402


def load_reference():
    for name in ("ignite_xdna", "ignite_xdna.compiler", "onnx", "onnx.numpy_helper"):
        if name not in sys.modules:
            mod = types.ModuleType(name)
            mod.__path__ = []
            sys.modules[name] = mod
    sys.modules["onnx"].numpy_helper = sys.modules["onnx.numpy_helper"]
    mods = {}
    for name in ("engine_emulator", "silu_sigmoid", "graph_ir", "graph_reference"):
        full = f"ignite_xdna.compiler.{name}"
        spec = importlib.util.spec_from_file_location(full, REF / "src/ignite_xdna/compiler" / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[full] = mod
        setattr(sys.modules["ignite_xdna.compiler"], name, mod)
        spec.loader.exec_module(mod)
        mods[name] = mod
    sys.path.insert(0, str(REF))     # tools/int4_prefill_model.py imports tools.xdna1_roofline
    try:
        import tools.int4_prefill_model as int4  # noqa: E402
    finally:
        sys.path.remove(str(REF))
    mods["int4"] = int4
    return mods


def to_reference_ir(ir, R):
    gi = R["graph_ir"]
    tensors = {n: gi.TensorInfo(t.name, t.channels, t.height, t.width, t.scale, t.zero_point, producer=t.producer)
               for n, t in ir.tensors.items()}
    layers = []
    for L in ir.layers:
        if isinstance(L, ConvLayer):
            segs = [gi.Segment(s.tensor, s.block_offset, s.blocks, s.up2) for s in L.inputs]
            rl = gi.ConvLayer(name=L.name, index=L.index, inputs=segs, in_scale=L.in_scale, k=L.k, stride=L.stride,
                              pad=L.pad, weights=L.weights, bias_q=L.bias_q, bias_scale=L.bias_scale,
                              weight_scale=L.weight_scale, conv_scale=L.conv_scale, output=L.output)
            if L.act is not None:
                rl.act = "silu_sigmoid"
                rl.act_scale = L.act_scale
                rl.sigmoid = R["silu_sigmoid"].fit_sigmoid(L.conv_scale, L.act_scale)
            if L.residual is not None:
                rl.residual = gi.Segment(L.residual.tensor, L.residual.block_offset, L.residual.blocks)
                rl.residual_shift = L.residual_shift
                rl.residual_lsh_main = L.residual_lsh_main
                rl.residual_lsh_res = L.residual_lsh_res
            layers.append(rl)
        else:
            layers.append(gi.PoolLayer(L.name, L.index, gi.Segment(L.input.tensor, L.input.block_offset,
                                                                    L.input.blocks), L.output))
    return gi.GraphIR(tensors=tensors, layers=layers, input=ir.input, outputs=list(ir.outputs),
                      silu_sigmoid=True, task=getattr(ir, "task", "detect"))


def ref_input(R, ir, pixels):
    scale = ir.tensors[ir.input].scale
    return R["graph_reference"].quantize_input(pixels.astype(np.float32) / np.float32(255.0), scale)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def fingerprint(ir) -> dict:
    layers = {}
    h = hashlib.sha256()
    for L in ir.layers:
        if isinstance(L, ConvLayer):
            d = hashlib.sha256()
            for a in (L.weights, L.bias_q):
                d.update(np.ascontiguousarray(a).tobytes())
            d.update(json.dumps([L.in_scale, L.weight_scale, L.conv_scale, L.act_scale, L.residual_shift,
                                 L.residual_lsh_main, L.residual_lsh_res]).encode())
            if L.sigmoid is not None:
                d.update(L.sigmoid.table.tobytes())
            layers[L.name] = d.hexdigest()
            h.update(d.digest())
    return {"model": h.hexdigest(), "layers": layers}


def make_kat(R, irs):
    em, ss = R["engine_emulator"], R["silu_sigmoid"]
    out = {}
    x = np.arange(-70000, 70000, dtype=np.int64)
    for s in (0, 1, 2, 5, 9, 12, 16):
        out[f"rne_{s}"] = em.rne_shift(x, s)
    tm, tr = np.meshgrid(np.arange(256), np.arange(256), indexing="ij")
    triples = {(0, 2, 2), (2, 0, 2), (1, 0, 0), (0, 0, 0), (0, 1, 1), (3, 0, 3)}
    for ir in irs:
        for L in ir.conv_layers():
            if L.residual is not None:
                triples.add((L.residual_lsh_main, L.residual_lsh_res, L.residual_shift))
    for a, b, s in sorted(triples):
        out[f"res_{a}_{b}_{s}"] = em.residual_combine(tm.astype(np.uint8), tr.astype(np.uint8), s, a, b)
    pairs = {(1 / 16, 1 / 32), (1 / 16, 1 / 16), (1 / 8, 1 / 16), (1 / 4, 1 / 4), (1 / 2, 1 / 2)}
    for ir in irs:
        for L in ir.conv_layers():
            if L.act is not None:
                pairs.add((L.conv_scale, L.act_scale))
    sig = []
    for s1, s2 in sorted(pairs):
        f = ss.fit_sigmoid(s1, s2)
        sig.append((s1, s2))
        out[f"sig_{s1!r}_{s2!r}_table"] = f.table
        out[f"sig_{s1!r}_{s2!r}_lines"] = np.array(f.params.lines, dtype=np.int64)
        out[f"sig_{s1!r}_{s2!r}_s_ysh"] = np.array([f.params.s, f.params.ysh], dtype=np.int64)
    out["sig_pairs"] = np.array(sig, dtype=np.float64)
    vals = np.arange(-8, 8, dtype=np.int8)
    out["int4_pack_range"] = R["int4"].Int4WeightPacker.pack(vals)
    out["int4_pack_3_m5"] = R["int4"].Int4WeightPacker.pack(np.array([3, -5], dtype=np.int8))
    rng = np.random.default_rng(1337)
    b = rng.integers(-8, 8, size=(64, 96), dtype=np.int8)
    out["int4_b"] = b
    out["int4_b_packed"] = R["int4"].Int4WeightPacker.pack(b)
    np.savez_compressed(HERE / "kat.npz", **out)


def make_small(R, imgsz, task="detect"):
    ir = build_yolov8("n", imgsz=imgsz, task=task)
    rir = to_reference_ir(ir, R)
    imgs = random_images(2, imgsz, seed=7)
    out = {"images": imgs}
    for i, im in enumerate(imgs):
        t = R["graph_reference"].run_direct(rir, ref_input(R, ir, im))
        for name, v in t.items():
            out[f"{i}|{name}"] = v
    tag = "_pose" if task == "pose" else ""
    np.savez_compressed(HERE / f"yolov8n{tag}_s{imgsz}.npz", **out)
    return ir


def hash_entry(R, ir):
    rir = to_reference_ir(ir, R)
    img = random_images(1, 640, seed=0)[0]
    t = R["graph_reference"].run_direct(rir, ref_input(R, ir, img))
    return {
        "spec": {k: v for k, v in ir.spec.items()},
        "fingerprint": fingerprint(ir),
        "image_seed": 0,
        "tensors": {name: sha(v) for name, v in t.items()},
        "heads": {hn: sha((t[tn].astype(np.int16) - 128).astype(np.int8)) for hn, tn in ir.outputs},
        "positions": {n: ti.scale for n, ti in ir.tensors.items()},
    }


def make_hashes(R):
    res = {}
    irs = []
    for variant in ("n", "s", "m"):
        ir = build_yolov8(variant, imgsz=640)
        irs.append(ir)
        res[f"yolov8{variant}"] = hash_entry(R, ir)
        print(f"yolov8{variant}: {len(res[f'yolov8{variant}']['tensors'])} tensors")
    with open(HERE / "graph_hashes.json", "w") as f:
        json.dump(res, f, indent=1, sort_keys=True)
    return irs


def make_pose(R):
    make_small(R, 64, task="pose")
    ir = build_yolov8("n", imgsz=640, task="pose")
    res = {"yolov8n-pose": hash_entry(R, ir)}
    with open(HERE / "pose_hashes.json", "w") as f:
        json.dump(res, f, indent=1, sort_keys=True)


def main():
    require_reference()
    R = load_reference()
    if "--pose" in sys.argv[1:]:
        make_pose(R)
        print("pose fixtures written to", HERE)
        return
    small = [make_small(R, 64), make_small(R, 96)]
    irs = make_hashes(R)
    make_kat(R, irs + small)
    make_pose(R)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
