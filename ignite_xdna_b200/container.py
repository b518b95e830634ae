"""The ``.ignite`` model container: reader, writer, and the B200 graph payload.

Container format (the reference's ``compiler/serializer.py``, layout :8-35, header :61-160,
writer :190-300, reader :308-447), restated here:

* a 64-byte little-endian header: magic ``IGNT``, format version (1), architecture id, header
  size (64), CRC-32 of every byte from offset 64 to the end, total size, manifest offset (64)
  and size, blob-section offset and size, blob count, 4 reserved bytes;
* the manifest, UTF-8 JSON (two-space indent), zero-padded to a multiple of 64 bytes; its
  ``blobs`` list is the directory: name, offset, size, content type and CRC-32 of each blob;
* the blobs, each at a 64-byte aligned offset, zero-padded to a multiple of 64 bytes.

The directory sits inside the manifest while the blob offsets depend on the manifest's padded
size, so the writer grows the padded size until the serialized manifest fits (as the reference's
writer does, :217-245); the reader checks every offset and size against the file before use.

The reference's containers carry an NPU graph (an XDNA ``xclbin``, instruction streams and AIE2
weight packets). This engine's containers carry the quantized graph itself, under the manifest
key ``b200_graph``: every tensor (shape, scale, zero point), every layer (the fields of the
reference's ``graph_ir.ConvLayer`` / ``PoolLayer``, :85-229) and, per conv, blobs for the
int8 weights [Cout][Cin][k][k], the int32 bias and, for a SiLU conv, the 256-byte table. The manifest
also keeps the reference's top-level keys a consumer of a detect container reads (``task``,
``input_shape``, ``quant_scales``, ``strides``, ``reg_max``, ``num_classes``, ``head_layout``,
``output_shapes``, ``egress_bytes``).
"""
from __future__ import annotations

import json
import mmap
import struct
import zlib
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple, Union

import numpy as np

from .graph import ConvLayer, GraphIR, PoolLayer, Segment, SigmoidFit, TensorInfo

MAGIC = b"IGNT"
FORMAT_VERSION = 1
ARCH_XDNA1 = 1       # the reference's NPU architectures
ARCH_XDNA2 = 2
ARCH_B200 = 0x10     # this engine's graph payload
ARCHS = (ARCH_XDNA1, ARCH_XDNA2, ARCH_B200)
HEADER = struct.Struct("<4sHHII5QI4s")
ALIGN = 64
assert HEADER.size == 64


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def _crc(b) -> int:
    return zlib.crc32(b) & 0xFFFFFFFF


# ---------------------------------------------------------------- container
def write_container(path: Union[str, Path], manifest: Dict[str, Any],
                    blobs: List[Tuple[str, bytes, str]], arch_id: int = ARCH_B200) -> int:
    """Write a container: ``blobs`` is [(name, data, content_type)]; returns the file size."""
    names = [n for n, _, _ in blobs]
    if len(set(names)) != len(names) or any(not n for n in names):
        raise ValueError("blob names must be unique and non-empty")
    base = {k: v for k, v in manifest.items() if k != "blobs"}
    crcs = [_crc(d) for _, d, _ in blobs]
    padded = _align(len(json.dumps(base, indent=2).encode()))
    for _ in range(64):
        off = HEADER.size + padded
        directory = []
        for (name, data, ctype), crc in zip(blobs, crcs):
            off = _align(off)
            directory.append({"name": name, "offset": off, "size": len(data), "content_type": ctype, "crc32": crc})
            off += _align(len(data))
        text = json.dumps(dict(base, blobs=directory), indent=2).encode()
        if _align(len(text)) <= padded:
            break
        padded = _align(len(text))
    else:
        raise RuntimeError("container layout did not settle")
    body = bytearray(text) + bytes(padded - len(text))
    for (name, data, _), ent in zip(blobs, directory):
        assert HEADER.size + len(body) == ent["offset"]
        body += data + bytes(_align(len(data)) - len(data))
    total = HEADER.size + len(body)
    blob_off = HEADER.size + padded
    head = HEADER.pack(MAGIC, FORMAT_VERSION, arch_id, HEADER.size, _crc(body), total, HEADER.size, len(text),
                       blob_off, total - blob_off, len(blobs), bytes(4))
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    with open(path, "wb") as f:
        f.write(head)
        f.write(body)
    return total


class Container:
    """A parsed container (memory-mapped when opened from a path): ``header``, ``manifest``,
    ``blob(name)`` as a zero-copy memoryview, ``verify()`` for the body and per-blob CRCs."""

    def __init__(self, src: Union[str, Path, bytes, bytearray]):
        self._file = self._map = None
        if isinstance(src, (str, Path)):
            self.path = Path(src)
            self._file = open(self.path, "rb")
            self._map = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
            self._buf = memoryview(self._map)
        else:
            self.path = None
            self._buf = memoryview(bytes(src))
        try:
            self._parse()
        except Exception:
            self.close()
            raise

    def _parse(self) -> None:
        n = len(self._buf)
        if n < HEADER.size:
            raise ValueError(f"container is {n} bytes, shorter than its 64-byte header")
        (magic, version, arch, hsize, crc, total, m_off, m_size, b_off, b_size, nblobs,
         _res) = HEADER.unpack(bytes(self._buf[:HEADER.size]))
        if magic != MAGIC:
            raise ValueError(f"not an .ignite container (magic {magic!r})")
        if hsize != HEADER.size or m_off != HEADER.size:
            raise ValueError("header size and manifest offset must both be 64")
        if version != FORMAT_VERSION:
            raise ValueError(f"unsupported container format version {version}")
        if arch not in ARCHS:
            raise ValueError(f"unknown architecture id {arch}")
        if total != n:
            raise ValueError(f"container declares {total} bytes but holds {n}")
        if m_off + m_size > n:
            raise ValueError("manifest runs past the end of the container")
        self.header = {"version": version, "arch_id": arch, "crc32": crc, "total_size": total,
                       "manifest_offset": m_off, "manifest_size": m_size, "blob_offset": b_off,
                       "blob_size": b_size, "num_blobs": nblobs}
        self.arch_id = arch
        self.manifest: Dict[str, Any] = json.loads(bytes(self._buf[m_off:m_off + m_size]).decode("utf-8"))
        self.blobs: Dict[str, Dict[str, Any]] = {}
        for e in self.manifest.get("blobs", []):
            name, off, size = e["name"], int(e["offset"]), int(e["size"])
            if name in self.blobs:
                raise ValueError(f"duplicate blob {name!r}")
            if off % ALIGN or off < m_off + m_size or size < 0 or off + size > n:
                raise ValueError(f"blob {name!r} [{off}, {off + size}) is misaligned or outside the blob section")
            self.blobs[name] = {"offset": off, "size": size, "content_type": e.get("content_type", "raw"),
                                "crc32": int(e.get("crc32", 0))}

    def blob(self, name: str) -> memoryview:
        if name not in self.blobs:
            raise KeyError(f"no blob {name!r} in the container")
        e = self.blobs[name]
        return self._buf[e["offset"]:e["offset"] + e["size"]]

    def verify(self) -> bool:
        """The body CRC of the header and every blob's CRC of the directory."""
        if _crc(self._buf[HEADER.size:]) != self.header["crc32"]:
            return False
        return all(_crc(self.blob(n)) == e["crc32"] for n, e in self.blobs.items())

    def close(self) -> None:
        if getattr(self, "_buf", None) is not None:
            try:
                self._buf.release()
            except (BufferError, ValueError):
                pass
            self._buf = None
        if self._map is not None:
            self._map.close()
            self._map = None
        if self._file is not None:
            self._file.close()
            self._file = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False


# ---------------------------------------------------------------- the B200 graph payload
def _seg(s: Optional[Segment]):
    return None if s is None else {"tensor": s.tensor, "block_offset": s.block_offset, "blocks": s.blocks,
                                   "up2": bool(s.up2)}


def _unseg(d) -> Optional[Segment]:
    return None if d is None else Segment(d["tensor"], int(d["block_offset"]), int(d["blocks"]), bool(d["up2"]))


def graph_manifest(ir: GraphIR, model_name: str = "") -> Tuple[Dict[str, Any], List[Tuple[str, bytes, str]]]:
    """The manifest and blobs of a container holding ``ir``."""
    tensors = {n: {"channels": t.channels, "height": t.height, "width": t.width, "scale": t.scale,
                   "zero_point": t.zero_point, "producer": t.producer} for n, t in ir.tensors.items()}
    layers, blobs = [], []
    i = -1
    for L in ir.layers:
        if isinstance(L, ConvLayer):
            i += 1
            d = {"kind": "conv", "name": L.name, "index": L.index, "inputs": [_seg(s) for s in L.inputs],
                 "in_scale": L.in_scale, "k": L.k, "stride": L.stride, "pad": L.pad,
                 "weights_shape": list(L.weights.shape), "bias_scale": L.bias_scale, "weight_scale": L.weight_scale,
                 "conv_scale": L.conv_scale, "output": L.output, "act": L.act, "residual": _seg(L.residual),
                 "residual_shift": L.residual_shift, "residual_lsh_main": L.residual_lsh_main,
                 "residual_lsh_res": L.residual_lsh_res, "act_scale": L.act_scale,
                 "weights": f"conv{i}.weights", "bias": f"conv{i}.bias", "table": None, "sigmoid": None}
            blobs.append((f"conv{i}.weights", np.ascontiguousarray(L.weights, dtype=np.int8).tobytes(), "int8"))
            blobs.append((f"conv{i}.bias", np.ascontiguousarray(L.bias_q, dtype=np.int32).tobytes(), "int32"))
            if L.sigmoid is not None:
                f = L.sigmoid
                d["table"] = f"conv{i}.table"
                d["sigmoid"] = {"lines": [list(map(int, ln)) for ln in f.lines], "s": int(f.s), "ysh": int(f.ysh),
                                "max_error": int(f.max_error), "mean_error": float(f.mean_error)}
                blobs.append((f"conv{i}.table", np.ascontiguousarray(f.table, dtype=np.uint8).tobytes(), "uint8"))
            layers.append(d)
        elif isinstance(L, PoolLayer):
            layers.append({"kind": "maxpool", "name": L.name, "index": L.index, "input": _seg(L.input),
                           "output": L.output, "k": L.k, "pad": L.pad})
        else:
            raise TypeError(f"layer {getattr(L, 'name', L)!r} has no container form")
    t_in = ir.tensors[ir.input]
    manifest: Dict[str, Any] = {
        "model_name": model_name, "format_version": FORMAT_VERSION, "arch_id": ARCH_B200,
        "target_hardware": "NVIDIA B200 (sm_100a)", "producer": "ignite_xdna_b200",
        "engine": "b200_xint8", "task": ir.task,
        "input_shape": [1, t_in.channels, t_in.height, t_in.width], "input_name": ir.input, "input_dtype": "uint8",
        "quant_scales": {"input_scale": t_in.scale, "input_zero_point": t_in.zero_point, "input_dtype": "uint8"},
        "b200_graph": {"tensors": tensors, "layers": layers, "input": ir.input,
                       "outputs": [[h, t] for h, t in ir.outputs], "silu_sigmoid": bool(ir.silu_sigmoid),
                       "spec": {k: v for k, v in ir.spec.items() if isinstance(v, (int, float, str, bool))}},
    }
    if ir.task in ("detect", "pose"):
        off, head_layout, shapes = 0, {}, {}
        for h, t in ir.outputs:
            ti = ir.tensors[t]
            head_layout[h] = {"offset": off, "scale": ti.scale, "zero_point": 0}
            shapes[h] = [1, ti.channels, ti.height, ti.width]
            off += ti.channels * ti.height * ti.width
        manifest.update({"strides": [8, 16, 32], "reg_max": ir.tensors[dict(ir.outputs)["p3_box"]].channels // 4,
                         "num_classes": ir.tensors[dict(ir.outputs)["p3_cls"]].channels, "fused_dfl": False,
                         "output_shapes": shapes, "head_layout": head_layout, "egress_bytes": off})
    return manifest, blobs


def save_container(ir: GraphIR, path: Union[str, Path], model_name: str = "") -> int:
    manifest, blobs = graph_manifest(ir, model_name)
    return write_container(path, manifest, blobs, ARCH_B200)


def graph_from_container(c: Container) -> GraphIR:
    """The GraphIR a container's ``b200_graph`` payload describes (checksums verified first)."""
    g = c.manifest.get("b200_graph")
    if g is None:
        if "graph_engine" in c.manifest:
            raise ValueError("this container holds an NPU graph-engine build (AIE2 instruction streams and weight "
                             "packets), not a quantized graph; write the graph itself with save_container")
        raise ValueError("the container's manifest has no b200_graph section")
    if not c.verify():
        raise ValueError("container checksum mismatch")
    tensors = {n: TensorInfo(n, int(t["channels"]), int(t["height"]), int(t["width"]), float(t["scale"]),
                             int(t["zero_point"]), t.get("producer", "")) for n, t in g["tensors"].items()}
    layers: List[object] = []
    for d in g["layers"]:
        if d["kind"] == "conv":
            w = np.frombuffer(c.blob(d["weights"]), dtype=np.int8).reshape(d["weights_shape"]).copy()
            b = np.frombuffer(c.blob(d["bias"]), dtype=np.int32).copy()
            if b.size != w.shape[0]:
                raise ValueError(f"{d['name']}: bias has {b.size} entries for {w.shape[0]} output channels")
            fit = None
            if d["sigmoid"] is not None:
                tab = np.frombuffer(c.blob(d["table"]), dtype=np.uint8).copy()
                if tab.size != 256:
                    raise ValueError(f"{d['name']}: activation table has {tab.size} entries")
                s = d["sigmoid"]
                fit = SigmoidFit(tuple(tuple(x) for x in s["lines"]), s["s"], s["ysh"], tab, s["max_error"],
                                 s["mean_error"])
            layers.append(ConvLayer(
                name=d["name"], index=int(d["index"]), inputs=[_unseg(s) for s in d["inputs"]],
                in_scale=float(d["in_scale"]), k=int(d["k"]), stride=int(d["stride"]), pad=int(d["pad"]),
                weights=w, bias_q=b, bias_scale=float(d["bias_scale"]), weight_scale=float(d["weight_scale"]),
                conv_scale=float(d["conv_scale"]), output=d["output"], act=d["act"], sigmoid=fit,
                residual=_unseg(d["residual"]), residual_shift=int(d["residual_shift"]),
                residual_lsh_main=int(d["residual_lsh_main"]),
                residual_lsh_res=None if d["residual_lsh_res"] is None else int(d["residual_lsh_res"]),
                act_scale=None if d["act_scale"] is None else float(d["act_scale"])))
        elif d["kind"] == "maxpool":
            layers.append(PoolLayer(d["name"], int(d["index"]), _unseg(d["input"]), d["output"], int(d["k"]),
                                    int(d["pad"])))
        else:
            raise ValueError(f"unknown layer kind {d['kind']!r}")
    return GraphIR(tensors=tensors, layers=layers, input=g["input"], outputs=[tuple(o) for o in g["outputs"]],
                   silu_sigmoid=bool(g.get("silu_sigmoid", True)), task=c.manifest.get("task", "detect"),
                   spec=dict(g.get("spec", {})))


def load_container(path: Union[str, Path]) -> GraphIR:
    with Container(path) as c:
        return graph_from_container(c)
