"""int4 expert weights on disk, and loading Hugging Face Mixtral checkpoints into the W4A16 layer.

Reference: python/light_moe/model/loader.py -- ``load_safetensors`` (:36-56) reads every
tensor of a ``.safetensors`` file; ``convert_hf_to_lightmoe`` (:72-140) maps the Mixtral
names, with the expert roles ``w1 -> gate_proj``, ``w3 -> up_proj``, ``w2 -> down_proj`` and
``block_sparse_moe.gate.weight -> moe.gate.gate.weight`` (:119-128); ``load_model_from_hf``
(:143-203) finds the weight files and the config (``MoEConfig.from_pretrained``,
config.py:71-104: ``num_local_experts``, ``num_experts_per_tok``, ``intermediate_size``).

Here only the MoE part of each decoder layer is read -- the router and the experts -- and
the experts are quantised to the library's int4 format on the GPU (symmetric, groups of
``group_size`` input values, fp16 scales; ``ops.quantize_w4``) and prepacked for the
W4A16 GEMMs.  The quantised weights can be saved as an int4 ``.safetensors`` file
(``save_w4a16`` / ``quantize_hf_mixtral``) and loaded back without re-quantising
(``load_w4a16``).

The safetensors container (an 8-byte little-endian header length, a JSON header mapping
each name to ``dtype`` / ``shape`` / ``data_offsets`` plus an optional ``__metadata__``
string map, then the raw little-endian tensor bytes) is read and written here directly, so
no extra package is needed; tensors are memory-mapped and copied to the device one at a
time.
"""
from __future__ import annotations

import json
import mmap
import os
import re
import struct
from typing import Dict, Iterable, Iterator, List, Optional, Tuple

import torch

from . import ops
from .layer import W4A16Experts, W4A16MoELayer

FORMAT = "light-moe-b200/w4a16"
FORMAT_VERSION = "1"

_DTYPES = {
    "BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32, "F64": torch.float64,
    "U8": torch.uint8, "I8": torch.int8, "I16": torch.int16, "I32": torch.int32, "I64": torch.int64,
    "BOOL": torch.bool,
}
_NAMES = {v: k for k, v in _DTYPES.items()}


# ------------------------------------------------------------------------------ container
class SafetensorsFile:
    """Read access to one ``.safetensors`` file (memory-mapped)."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        if size < 8:
            raise ValueError(f"{path}: not a safetensors file")
        (n,) = struct.unpack("<Q", self._f.read(8))
        if n > size - 8:
            raise ValueError(f"{path}: header length {n} exceeds the file")
        header = json.loads(self._f.read(n).decode("utf-8"))
        self.metadata: Dict[str, str] = header.pop("__metadata__", {}) or {}
        self.entries: Dict[str, dict] = header
        self._base = 8 + n
        self._map = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_COPY) if size > self._base else None
        for name, e in self.entries.items():
            b, en = e["data_offsets"]
            if e["dtype"] not in _DTYPES or not 0 <= b <= en <= size - self._base:
                raise ValueError(f"{path}: bad entry {name}")

    def keys(self) -> List[str]:
        return list(self.entries)

    def shape(self, name: str) -> Tuple[int, ...]:
        return tuple(self.entries[name]["shape"])

    def get(self, name: str) -> torch.Tensor:
        """The tensor (CPU; shares the file mapping until copied)."""
        e = self.entries[name]
        dt = _DTYPES[e["dtype"]]
        b, en = e["data_offsets"]
        shape = tuple(e["shape"])
        if en == b:
            return torch.empty(shape, dtype=dt)
        buf = memoryview(self._map)[self._base + b:self._base + en]
        return torch.frombuffer(buf, dtype=torch.uint8).view(dt).reshape(shape)

    def close(self):
        if self._map is not None:
            self._map.close()
            self._map = None
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def write_safetensors(path: str, tensors: Dict[str, torch.Tensor], metadata: Optional[Dict[str, str]] = None):
    """Write ``tensors`` (any device; copied to the host) as a ``.safetensors`` file."""
    header = {}
    blobs = []
    off = 0
    for name, t in tensors.items():
        if t.dtype not in _NAMES:
            raise ValueError(f"{name}: dtype {t.dtype} has no safetensors code")
        raw = t.detach().to("cpu").contiguous().view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)   # the data starts 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for raw in blobs:
            f.write(raw)


# ------------------------------------------------------------------------------ Mixtral checkpoints
_EXPERT_RE = re.compile(r"^model\.layers\.(\d+)\.block_sparse_moe\.experts\.(\d+)\.(w[123])\.weight$")
_GATE_RE = re.compile(r"^model\.layers\.(\d+)\.block_sparse_moe\.gate\.weight$")
# the reference's role map (loader.py:123-128): w1 = gate_proj, w3 = up_proj, w2 = down_proj
ROLES = {"w1": "gate_proj", "w3": "up_proj", "w2": "down_proj"}


def read_hf_config(model_dir: str) -> dict:
    """The MoE sizes of a Hugging Face Mixtral ``config.json`` (keys as MoEConfig.from_pretrained
    reads them, config.py:91-104)."""
    with open(os.path.join(model_dir, "config.json")) as f:
        c = json.load(f)
    return {"hidden_size": int(c.get("hidden_size", 4096)), "intermediate_size": int(c.get("intermediate_size", 14336)),
            "num_experts": int(c.get("num_local_experts", 8)), "top_k": int(c.get("num_experts_per_tok", 2)),
            "num_layers": int(c.get("num_hidden_layers", 32))}


def hf_weight_files(model_dir: str) -> List[str]:
    """The checkpoint's ``.safetensors`` shards (from ``model.safetensors.index.json`` when present)."""
    idx = os.path.join(model_dir, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(model_dir, p) for p in files]
    files = sorted(p for p in os.listdir(model_dir) if p.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {model_dir}")
    return [os.path.join(model_dir, p) for p in files]


def moe_tensor_index(files: Iterable[str]) -> Dict[int, dict]:
    """Per decoder layer, where its router and expert tensors live:
    ``{layer: {"gate": (file, name), ("w1", e): (file, name), ...}}``."""
    index: Dict[int, dict] = {}
    for path in files:
        with SafetensorsFile(path) as st:
            for name in st.keys():
                m = _EXPERT_RE.match(name)
                if m:
                    index.setdefault(int(m.group(1)), {})[(m.group(3), int(m.group(2)))] = (path, name)
                    continue
                m = _GATE_RE.match(name)
                if m:
                    index.setdefault(int(m.group(1)), {})["gate"] = (path, name)
    return index


def _read(path_name, cache: Dict[str, SafetensorsFile]) -> torch.Tensor:
    path, name = path_name
    if path not in cache:
        cache[path] = SafetensorsFile(path)
    return cache[path].get(name)


def iter_hf_moe_layers(model_dir: str, layers: Optional[Iterable[int]] = None) -> Iterator[Tuple[int, dict]]:
    """Yield ``(layer, {"gate": [E, d], "w1": [E, ffn, d], "w3": [E, ffn, d], "w2": [E, d, ffn]})``
    (CPU tensors in the checkpoint's dtype) for the MoE layers of a Mixtral checkpoint."""
    cfg = read_hf_config(model_dir)
    index = moe_tensor_index(hf_weight_files(model_dir))
    want = sorted(index) if layers is None else list(layers)
    cache: Dict[str, SafetensorsFile] = {}
    try:
        for li in want:
            entry = index.get(li)
            if entry is None or "gate" not in entry:
                raise KeyError(f"layer {li}: no block_sparse_moe tensors in the checkpoint")
            E = cfg["num_experts"]
            missing = [(r, e) for r in ROLES for e in range(E) if (r, e) not in entry]
            if missing:
                raise KeyError(f"layer {li}: missing expert tensors {missing[:4]}")
            out = {"gate": _read(entry["gate"], cache).clone()}
            for r in ROLES:
                out[r] = torch.stack([_read(entry[(r, e)], cache) for e in range(E)])
            yield li, out
    finally:
        for st in cache.values():
            st.close()


# ------------------------------------------------------------------------------ int4 file
def _quantize_layer(w: dict, group_size: int, device) -> dict:
    """Quantise one layer's experts on ``device`` expert by expert (bounded transient memory)."""
    out = {"gate": w["gate"].to(device=device, dtype=torch.bfloat16)}
    for r in ROLES:
        qs, ss = [], []
        for e in range(w[r].shape[0]):
            q, s = ops.quantize_w4(w[r][e].to(device=device, dtype=torch.bfloat16), group_size)
            qs.append(q)
            ss.append(s)
        out[r + ".qweight"] = torch.stack(qs)
        out[r + ".scales"] = torch.stack(ss)
    return out


def _layer_from_int4(t: dict, top_k: int, group_size: int) -> W4A16MoELayer:
    E = t["gate"].shape[0]
    ex = W4A16Experts.from_quantized(t["w1.qweight"], t["w1.scales"], t["w3.qweight"], t["w3.scales"],
                                     t["w2.qweight"], t["w2.scales"], E, group_size, keep_canonical=True)
    return W4A16MoELayer(t["gate"], ex, top_k)


def quantize_hf_mixtral(model_dir: str, out_path: str, group_size: int = 128, layers: Optional[Iterable[int]] = None,
                        device=None) -> dict:
    """Read a Mixtral checkpoint's MoE layers, quantise their experts to int4 on the GPU and
    write them as one int4 ``.safetensors`` file (names ``layers.{i}.gate.weight`` bf16 [E, d],
    ``layers.{i}.{w1,w3,w2}.qweight`` uint8 [E, rows, K/2] and ``.scales`` fp16
    [E, rows, K/group_size], in the canonical int4 format).  Returns the file's metadata."""
    cfg = read_hf_config(model_dir)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    tensors: Dict[str, torch.Tensor] = {}
    done = []
    for li, w in iter_hf_moe_layers(model_dir, layers):
        for name, t in _quantize_layer(w, group_size, dev).items():
            tensors[f"layers.{li}.{name}" if name != "gate" else f"layers.{li}.gate.weight"] = t
        done.append(li)
    meta = {"format": FORMAT, "version": FORMAT_VERSION, "group_size": group_size, "num_experts": cfg["num_experts"],
            "top_k": cfg["top_k"], "hidden_size": cfg["hidden_size"], "ffn_size": cfg["intermediate_size"],
            "layers": ",".join(str(i) for i in done)}
    write_safetensors(out_path, tensors, meta)
    return {k: str(v) for k, v in meta.items()}


def save_w4a16(path: str, layers: Dict[int, W4A16MoELayer]):
    """Write layers built with ``keep_canonical=True`` (e.g. by ``load_hf_mixtral_moe``) as an
    int4 ``.safetensors`` file readable by ``load_w4a16``."""
    tensors: Dict[str, torch.Tensor] = {}
    meta = None
    for li, layer in sorted(layers.items()):
        ex = layer.experts
        if ex.canonical is None:
            raise ValueError(f"layer {li}: built without canonical int4 copies (keep_canonical=True)")
        if ex.num_shared:
            raise ValueError("shared experts are not part of the Mixtral format")
        c = ex.canonical
        tensors[f"layers.{li}.gate.weight"] = layer.gate_weight
        for r, (q, s) in (("w1", ("q1", "s1")), ("w3", ("q3", "s3")), ("w2", ("q2", "s2"))):
            tensors[f"layers.{li}.{r}.qweight"] = c[q]
            tensors[f"layers.{li}.{r}.scales"] = c[s]
        m = {"format": FORMAT, "version": FORMAT_VERSION, "group_size": ex.group_size, "num_experts": ex.num_experts,
             "top_k": layer.top_k, "hidden_size": ex.hidden_size, "ffn_size": ex.ffn_size}
        if meta is not None and any(meta[k] != m[k] for k in m):
            raise ValueError("layers of different shapes cannot share one file")
        meta = m
    if meta is None:
        raise ValueError("no layers")
    meta["layers"] = ",".join(str(i) for i in sorted(layers))
    write_safetensors(path, tensors, meta)


def load_w4a16(path: str, device=None, layers: Optional[Iterable[int]] = None) -> Dict[int, W4A16MoELayer]:
    """Load an int4 file written by ``quantize_hf_mixtral`` / ``save_w4a16``: one
    ``W4A16MoELayer`` per stored layer (prepacked on ``device``)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    with SafetensorsFile(path) as st:
        meta = st.metadata
        if meta.get("format") != FORMAT:
            raise ValueError(f"{path}: not a {FORMAT} file (format={meta.get('format')!r})")
        if meta.get("version") != FORMAT_VERSION:
            raise ValueError(f"{path}: format version {meta.get('version')!r} is not {FORMAT_VERSION}")
        g, top_k = int(meta["group_size"]), int(meta["top_k"])
        stored = [int(i) for i in meta["layers"].split(",") if i != ""]
        want = stored if layers is None else list(layers)
        out = {}
        for li in want:
            if li not in stored:
                raise KeyError(f"layer {li} is not in {path}")
            t = {"gate": st.get(f"layers.{li}.gate.weight").to(dev)}
            for r in ROLES:
                for part in ("qweight", "scales"):
                    t[f"{r}.{part}"] = st.get(f"layers.{li}.{r}.{part}").to(dev)
            out[li] = _layer_from_int4(t, top_k, g)
        return out


def load_hf_mixtral_moe(model_dir: str, group_size: int = 128, layers: Optional[Iterable[int]] = None,
                        device=None) -> Dict[int, W4A16MoELayer]:
    """A Mixtral checkpoint's MoE layers as ``W4A16MoELayer`` objects, quantised on the fly
    (``keep_canonical=True``, so ``save_w4a16`` can write them)."""
    cfg = read_hf_config(model_dir)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    return {li: _layer_from_int4(_quantize_layer(w, group_size, dev), cfg["top_k"], group_size)
            for li, w in iter_hf_moe_layers(model_dir, layers)}
