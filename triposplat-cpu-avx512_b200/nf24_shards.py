"""NF24 shard directories (format ``triposplat_nf24_i16_v1``) loaded straight into device memory.

The reference keeps a packed checkpoint as a directory
(``scripts/native_linear_nf24_prepacked.py:202-335``): ``manifest.json`` (format, complete
flag, residual mode, source checkpoint identity, per-Linear file / sha256 / bytes / shape /
bias flag / quantisation report, the non-Linear file), one safetensors file per Linear
holding ``code01_t`` int16 [in, out], ``q2_t`` int8 [in, out], ``scale`` f32 [out] and
``bias`` f32 [out], and ``non_linear.safetensors`` with every other tensor.  Its loader
(``:338-437``) builds the model on the meta device and registers the code tensors as CPU
buffers.

``load_nf24_shards`` reads the same directory into GPU memory: manifest checks as the
reference's loader (format, complete, nf24_i16, shapes), optional sha256 verification run
on a thread pool while the files are read, each file's tensors copied to the device once,
and optionally the k-contiguous code planes (``triposplat_b200_nf24_codes_to_nk``) the
split GEMMs read.  ``save_nf24_shards`` writes the same format from packed weights (file
names, manifest fields and JSON layout as the reference's packer), so shards move both ways.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import json
import os
from dataclasses import dataclass, field
from pathlib import Path

FORMAT = "triposplat_nf24_i16_v1"


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as f:
        for chunk in iter(lambda: f.read(8 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _linear_filename(index: int, name: str) -> str:
    return f"linears/{index:03d}_{hashlib.sha256(name.encode('utf-8')).hexdigest()[:12]}.safetensors"


def _write_json(path: Path, value) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(value, indent=2, sort_keys=True) + "\n")
    os.replace(tmp, path)


@dataclass
class ShardLinear:
    code01: object        # int16 [in, out], on the device
    q2: object            # int8  [in, out]
    scale: object         # f32 [out]
    bias: object          # f32 [out]
    has_bias: bool = True
    code01_nk: object = None  # int16 [out, in] (with nk=True)
    q2_nk: object = None      # int8  [out, in]


@dataclass
class ShardSet:
    manifest: dict
    linears: dict = field(default_factory=dict)     # name -> ShardLinear
    non_linear: dict = field(default_factory=dict)  # name -> tensor on the device
    loaded_bytes: int = 0
    checksums_verified: bool = False


def read_manifest(root) -> dict:
    root = Path(root)
    manifest = json.loads((root / "manifest.json").read_text())
    if manifest.get("format") != FORMAT or not manifest.get("complete"):
        raise RuntimeError(f"invalid or incomplete NF24 checkpoint: {root}")
    if manifest.get("residual_mode") != "nf24_i16":
        raise RuntimeError("prepacked checkpoint is not NF24 int16")
    return manifest


def load_nf24_shards(root, device: str = "cuda", *, verify_checksums: bool = False,
                     nk: bool = False, names=None, workers: int = 8) -> ShardSet:
    """Load a shard directory into `device` memory.

    verify_checksums: sha256 of every file against the manifest (on `workers` threads,
    overlapping the reads); a mismatch raises.  nk: also build the k-contiguous code
    planes on the device.  names: load only these Linears (all by default).
    """
    import torch
    from safetensors.torch import load_file

    root = Path(root)
    manifest = read_manifest(root)
    items = manifest["linears"]
    wanted = list(items) if names is None else list(names)
    missing = [n for n in wanted if n not in items]
    if missing:
        raise RuntimeError(f"linears not in the manifest: {missing}")
    out = ShardSet(manifest=manifest, checksums_verified=bool(verify_checksums))
    files = [(n, root / items[n]["file"], items[n]) for n in wanted]
    nl = manifest["non_linear"]
    with cf.ThreadPoolExecutor(max_workers=max(1, workers)) as pool:
        sums = {}
        if verify_checksums:
            sums = {n: pool.submit(_sha256, p) for n, p, _ in files}
            sums["__non_linear__"] = pool.submit(_sha256, root / nl["file"])
        reads = {n: pool.submit(load_file, p.as_posix(), "cpu") for n, p, _ in files}
        for n, path, item in files:
            t = reads[n].result()
            shape = (int(item["in_features"]), int(item["out_features"]))
            if tuple(t["code01_t"].shape) != shape or tuple(t["q2_t"].shape) != shape:
                raise RuntimeError(f"packed shape mismatch for {n}")
            if t["code01_t"].dtype != torch.int16 or t["q2_t"].dtype != torch.int8:
                raise RuntimeError(f"packed dtype mismatch for {n}")
            if verify_checksums and sums[n].result() != item["sha256"]:
                raise RuntimeError(f"checksum mismatch: {path}")
            dev = {k: v.to(device, non_blocking=False) for k, v in t.items()}
            out.linears[n] = ShardLinear(dev["code01_t"], dev["q2_t"], dev["scale"], dev["bias"],
                                         bool(item.get("has_bias", True)))
            out.loaded_bytes += int(item["bytes"])
        if verify_checksums and sums["__non_linear__"].result() != nl["sha256"]:
            raise RuntimeError(f"checksum mismatch: {root / nl['file']}")
    out.non_linear = {k: v.to(device) for k, v in load_file((root / nl["file"]).as_posix(), "cpu").items()}
    out.loaded_bytes += int(nl["bytes"])
    if nk:
        import _native

        lib = _native.load()
        _native.use_current_stream(lib)
        for n, lin in out.linears.items():
            K, N = (int(d) for d in lin.code01.shape)
            lin.code01_nk = torch.empty(N, K, dtype=torch.int16, device=device)
            lin.q2_nk = torch.empty(N, K, dtype=torch.int8, device=device)
            st = lib.triposplat_b200_nf24_codes_to_nk(lin.code01.data_ptr(), lin.q2.data_ptr(), K, N,
                                                      lin.code01_nk.data_ptr(), lin.q2_nk.data_ptr())
            if st:
                raise RuntimeError(f"codes_to_nk returned {st} for {n}")
    return out


def save_nf24_shards(linears: dict, out_dir, *, non_linear: dict | None = None,
                     source: dict | None = None, quantization: dict | None = None,
                     has_bias: dict | None = None) -> dict:
    """Write packed Linears (name -> object with code01 / q2 / scale / bias tensors) and the
    non-Linear tensors as a ``triposplat_nf24_i16_v1`` directory; returns the manifest.
    Linears are numbered in the sorted order of their "<name>.weight" keys, as the
    reference's packer numbers the sorted checkpoint keys."""
    import torch
    from safetensors.torch import save_file

    root = Path(out_dir)
    (root / "linears").mkdir(parents=True, exist_ok=True)
    manifest = {
        "format": FORMAT, "complete": False, "residual_mode": "nf24_i16", "bits_per_weight": 24,
        "source": source or {"name": "in-memory", "bytes": 0, "sha256": ""},
        "linear_count": len(linears), "linears": {},
    }
    for index, name in enumerate(sorted(linears, key=lambda n: n + ".weight")):
        lin = linears[name]
        rel = _linear_filename(index, name)
        target = root / rel
        tensors = {k: getattr(lin, a).detach().to("cpu").contiguous() for k, a in
                   (("code01_t", "code01"), ("q2_t", "q2"), ("scale", "scale"), ("bias", "bias"))}
        if tensors["code01_t"].dtype != torch.int16 or tensors["q2_t"].dtype != torch.int8:
            raise ValueError(f"{name}: code01 must be int16 and q2 int8")
        tmp = target.with_suffix(target.suffix + ".tmp")
        save_file(tensors, tmp.as_posix())
        os.replace(tmp, target)
        K, N = (int(d) for d in tensors["code01_t"].shape)
        manifest["linears"][name] = {
            "file": rel, "sha256": _sha256(target), "bytes": target.stat().st_size,
            "in_features": K, "out_features": N,
            "has_bias": bool((has_bias or {}).get(name, True)), "weight_elements": K * N,
            "quantization": (quantization or {}).get(name, {"residual_mode": "nf24_i16"}),
        }
    nl_path = root / "non_linear.safetensors"
    nl = {k: v.detach().to("cpu", dtype=torch.float32).contiguous() for k, v in (non_linear or {}).items()}
    tmp = nl_path.with_suffix(nl_path.suffix + ".tmp")
    save_file(nl, tmp.as_posix())
    os.replace(tmp, nl_path)
    manifest["non_linear"] = {"file": nl_path.name, "sha256": _sha256(nl_path),
                              "bytes": nl_path.stat().st_size, "tensor_count": len(nl)}
    manifest["packed_bytes"] = sum(i["bytes"] for i in manifest["linears"].values()) + \
        manifest["non_linear"]["bytes"]
    manifest["complete"] = True
    _write_json(root / "manifest.json", manifest)
    return manifest


def save_flow_weights(weights, out_dir) -> dict:
    """The synthetic flow model's packed weights (flow_model.FlowWeights) as a shard
    directory: every Linear as an NF24 file, the per-block tables and gammas as the
    non-Linear tensors."""
    return save_nf24_shards(weights.linears, out_dir, non_linear=weights.params)


def load_flow_weights(root, spec, device: str = "cuda", *, verify_checksums: bool = False):
    """flow_model.FlowWeights for `spec` read from a shard directory into `device` memory;
    the Linear set must be exactly spec.linears()."""
    from flow_model import FlowWeights, PackedLinear

    sh = load_nf24_shards(root, device, verify_checksums=verify_checksums)
    want = {name: (k, n) for name, k, n in spec.linears()}
    if set(sh.linears) != set(want):
        raise RuntimeError("shard Linears do not match the model spec: "
                           f"missing={sorted(set(want) - set(sh.linears))} "
                           f"extra={sorted(set(sh.linears) - set(want))}")
    w = FlowWeights(spec)
    for name, (k, n) in want.items():
        lin = sh.linears[name]
        if tuple(lin.code01.shape) != (k, n):
            raise RuntimeError(f"{name}: shard shape {tuple(lin.code01.shape)} != {(k, n)}")
        w.linears[name] = PackedLinear(lin.code01, lin.q2, lin.scale, lin.bias)
    w.params = dict(sh.non_linear)
    return w


def _entry_valid(root: Path, item) -> bool:
    if not item or "file" not in item or "sha256" not in item:
        return False
    path = root / item["file"]
    return path.is_file() and path.stat().st_size == item.get("bytes") and _sha256(path) == item["sha256"]


def pack_nf24_i16_checkpoint(source_checkpoint, output_dir, *, expected_linear_count: int = 206,
                             device: str = "cpu") -> dict:
    """A safetensors checkpoint packed into a ``triposplat_nf24_i16_v1`` directory, under the
    reference packer's name and contract (scripts/native_linear_nf24_prepacked.py:202-335):
    every 2-D ``*.weight`` tensor is a Linear (their count must equal
    ``expected_linear_count``), packed by this package's NF24 packer (bit-identical codes;
    ``device`` selects where the packing runs); a missing bias packs as zeros; every other
    tensor goes to ``non_linear.safetensors``.  A directory already complete for the same
    source checkpoint (name, size, sha256) is returned unchanged."""
    import torch
    from safetensors import safe_open

    from nf24_pack import make_nf8_codebook, quantize_nf24_i16_any_device

    source = Path(source_checkpoint).resolve()
    root = Path(output_dir).resolve()
    source_info = {"name": source.name, "bytes": source.stat().st_size, "sha256": _sha256(source)}
    manifest_path = root / "manifest.json"
    if manifest_path.is_file():
        existing = json.loads(manifest_path.read_text())
        if existing.get("format") != FORMAT or existing.get("source") != source_info:
            raise RuntimeError("existing prepacked manifest does not match source checkpoint")
        if (existing.get("complete") and all(_entry_valid(root, i) for i in existing["linears"].values())
                and _entry_valid(root, existing.get("non_linear"))):
            return existing
    codebook = make_nf8_codebook(torch)
    with safe_open(source.as_posix(), framework="pt", device="cpu") as handle:
        keys = sorted(handle.keys())
        weight_keys = [k for k in keys if k.endswith(".weight") and len(handle.get_slice(k).get_shape()) == 2]
        if len(weight_keys) != expected_linear_count:
            raise RuntimeError(f"expected {expected_linear_count} Linear weights, found {len(weight_keys)}")
        names = [k[:-7] for k in weight_keys]
        linear_keys = set(weight_keys) | {f"{n}.bias" for n in names if f"{n}.bias" in keys}
        packed, quant, has_bias = {}, {}, {}
        for name, wkey in zip(names, weight_keys):
            weight = handle.get_tensor(wkey).to(torch.float32).contiguous().to(device)
            codes, scales, error = quantize_nf24_i16_any_device(weight, codebook)
            bkey = f"{name}.bias"
            has_bias[name] = bkey in keys
            bias = (handle.get_tensor(bkey).to(torch.float32).contiguous() if has_bias[name]
                    else torch.zeros(weight.shape[0], dtype=torch.float32))

            class _P:  # the attribute layout save_nf24_shards reads
                pass
            p = _P()
            p.code01, p.q2, p.scale, p.bias = codes[0].cpu(), codes[1].cpu(), scales[0].cpu(), bias
            packed[name] = p
            quant[name] = error
        non_linear = {k: handle.get_tensor(k).to(torch.float32).contiguous() for k in keys if k not in linear_keys}
    return save_nf24_shards(packed, root, non_linear=non_linear, source=source_info, quantization=quant,
                            has_bias=has_bias)


def load_nf24_i16_prepacked_model(packed_dir, model_factory, *, verify_checksums: bool = False,
                                  device: str = "cuda"):
    """Build ``model_factory()`` with its Linear parameters on the meta device and fill it
    from a shard directory, under the reference loader's name and contract
    (scripts/native_linear_nf24_prepacked.py:359-437): the model's Linear set must equal the
    manifest's, the non-Linear state must account for every other parameter, each Linear
    gets the ``_native_rnf8_*`` buffers the NF24 patch reads and empty float weights, and
    the model carries ``_native_rnf8_prepacked_manifest`` / ``_native_rnf8_prepacked_load``.
    Everything lands on ``device`` (the reference: the host); the source checkpoint is
    never read."""
    import torch
    import torch.nn as nn

    original = nn.Linear.__init__

    def on_meta(module, in_features, out_features, bias=True, device=None, dtype=None):
        return original(module, in_features, out_features, bias=bias, device="meta", dtype=dtype)

    nn.Linear.__init__ = on_meta
    try:
        model = model_factory()
    finally:
        nn.Linear.__init__ = original
    linears = {n: m for n, m in model.named_modules() if isinstance(m, nn.Linear)}
    manifest = read_manifest(packed_dir)
    if set(linears) != set(manifest["linears"]):
        raise RuntimeError("prepacked/model Linear mismatch: "
                           f"missing={sorted(set(linears) - set(manifest['linears']))} "
                           f"extra={sorted(set(manifest['linears']) - set(linears))}")
    shards = load_nf24_shards(packed_dir, device, verify_checksums=verify_checksums)
    incompatible = model.load_state_dict(shards.non_linear, strict=False, assign=True)
    expected_missing = {f"{n}.{f}" for n, m in linears.items()
                        for f in (("weight", "bias") if m.bias is not None else ("weight",))}
    if set(incompatible.missing_keys) != expected_missing or incompatible.unexpected_keys:
        raise RuntimeError("non-Linear state mismatch: "
                           f"missing={incompatible.missing_keys} unexpected={incompatible.unexpected_keys}")
    for name, module in linears.items():
        lin = shards.linears[name]
        module.register_buffer("_native_rnf8_codes0_t", lin.code01, persistent=False)
        module.register_buffer("_native_rnf8_codes1_t", lin.q2, persistent=False)
        module.register_buffer("_native_rnf8_codes2_t", lin.q2, persistent=False)
        module.register_buffer("_native_rnf8_scales0", lin.scale, persistent=False)
        module.register_buffer("_native_rnf8_scales1", lin.scale, persistent=False)
        module.register_buffer("_native_rnf8_scales2", lin.scale, persistent=False)
        module.register_buffer("_native_rnf8_bias", lin.bias, persistent=False)
        module.weight = nn.Parameter(torch.empty(0, dtype=torch.float32, device=device), requires_grad=False)
        if module.bias is not None:
            module.bias = nn.Parameter(torch.empty(0, dtype=torch.float32, device=device), requires_grad=False)
    model._native_rnf8_prepacked_manifest = manifest
    model._native_rnf8_prepacked_load = {
        "enabled": True, "format": FORMAT, "directory": Path(packed_dir).resolve().as_posix(),
        "linear_count": len(linears), "loaded_bytes": shards.loaded_bytes,
        "checksums_verified": bool(verify_checksums), "source_checkpoint_loaded": False,
        "device": str(device),
    }
    return model
