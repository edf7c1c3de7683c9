"""Packed-record artefact on disk: the neuron-major records plus a versioned manifest.

The reference writes an optional runtime artefact with gate, up and a
transposed down as three separate safetensors tensors
(runtime/weights.py:89-96, ``save_neuron_major_layout``; CLI
scripts/pack_neuron_major_weights.py), and keeps its low-VRAM stream cache
behind a versioned manifest whose payload files carry byte sizes and sha256
digests (integration/freetoken_qcc/low_vram/manifest.py:9-57).  Here one
directory holds:

* ``records.bin`` -- the packed records exactly as they sit in HBM,
  ``[N, 3 * Hp]`` in the layer's dtype, record n = [gate[n] | up[n] | down[:, n]]
  zero padded to Hp = hidden rounded up to 8 (the layout of
  ``qcc_pack_records``), so loading is one copy with no re-packing, a shard
  reads only its contiguous rows, and the host-offload store can map it;
* ``manifest.json`` -- format name and version, dtype, hidden, Hp,
  intermediate, record bytes, and the payload's byte size and sha256.

``load_manifest`` refuses unknown formats or versions and missing or
inconsistent fields; ``validate_files`` checks the payload's size and,
optionally, its digest.  The errors are ``FileNotFoundError`` for a missing
file and ``ValueError`` otherwise, as in the reference's manifest checks.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch

from .packing import PackedFFNWeights, validate_weight_shapes

FORMAT = "qcc-b200-packed-records"
FORMAT_VERSION = 1
LAYOUT = "neuron-major [gate | up | down] records, zero padded to hidden_pad"
RECORDS_FILE = "records.bin"
MANIFEST_FILE = "manifest.json"
ROLES = ("gate_proj.weight", "up_proj.weight", "down_proj.weight")  # reference runtime/weights.py:15

_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
_CHUNK = 64 << 20


def _dtype_name(dtype: torch.dtype) -> str:
    for name, value in _DTYPES.items():
        if value == dtype:
            return name
    raise TypeError(f"unsupported record dtype {dtype}")


def file_sha256(path: Path, chunk_size: int = _CHUNK) -> str:
    digest = hashlib.sha256()
    with Path(path).open("rb") as handle:
        for chunk in iter(lambda: handle.read(chunk_size), b""):
            digest.update(chunk)
    return digest.hexdigest()


def pack_records_host(gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor,
                      transposed_down: bool = False) -> torch.Tensor:
    """The packed ``[N, 3 * Hp]`` records of three host tensors, for writing an artefact.

    Layout tooling, run once per layer: on a GPU the same records come from
    ``pack_neuron_major`` (``qcc_pack_records``), which ``write_artefact``
    uses whenever the weights are already on a CUDA device.
    """
    hidden, n = validate_weight_shapes(gate, up, down, transposed_down)
    if gate.dtype != up.dtype or gate.dtype != down.dtype:
        raise TypeError("gate, up and down must share a dtype")
    hp = (hidden + 7) // 8 * 8
    packed = torch.zeros((n, 3 * hp), dtype=gate.dtype)
    packed[:, :hidden] = gate
    packed[:, hp:hp + hidden] = up
    packed[:, 2 * hp:2 * hp + hidden] = down if transposed_down else down.t()
    return packed


def write_artefact(root: Path | str, weights, *, source: str | None = None, metadata: dict | None = None) -> dict:
    """Write a packed layer (``PackedFFNWeights``, or ``(gate, up, down)``) to ``root``; returns the manifest.

    The records are streamed to disk in chunks and hashed on the way.
    """
    from .packing import pack_neuron_major

    if isinstance(weights, PackedFFNWeights):
        packed, hidden = weights.packed, weights.hidden
        offset, total = weights.record_offset, weights.intermediate
    else:
        gate, up, down = weights
        if gate.is_cuda:
            pw = pack_neuron_major(gate, up, down)
            packed, hidden, offset, total = pw.packed, pw.hidden, 0, pw.intermediate
        else:
            packed = pack_records_host(gate, up, down)
            hidden, offset, total = gate.shape[1], 0, gate.shape[0]
    root = Path(root)
    root.mkdir(parents=True, exist_ok=True)
    n, width = packed.shape
    hp = (hidden + 7) // 8 * 8
    if width != 3 * hp:
        raise ValueError(f"packed records have width {width}, expected 3 * {hp}")
    digest = hashlib.sha256()
    path = root / RECORDS_FILE
    rows_per_chunk = max(1, _CHUNK // max(1, width * packed.element_size()))
    with path.open("wb") as handle:
        for start in range(0, n, rows_per_chunk):
            rows = packed[start:start + rows_per_chunk].detach().to("cpu").contiguous()
            raw = rows.view(torch.uint8).numpy().tobytes()
            digest.update(raw)
            handle.write(raw)
    manifest = {
        "format": FORMAT,
        "format_version": FORMAT_VERSION,
        "layout": LAYOUT,
        "dtype": _dtype_name(packed.dtype),
        "hidden": int(hidden),
        "hidden_pad": int(hp),
        "intermediate": int(n),
        "record_offset": int(offset),
        "total_intermediate": int(total),
        "record_bytes": int(3 * hp * packed.element_size()),
        "records": {"file": RECORDS_FILE, "file_bytes": int(path.stat().st_size), "sha256": digest.hexdigest()},
        "source": source,
        "metadata": dict(metadata or {}),
    }
    (root / MANIFEST_FILE).write_text(json.dumps(manifest, indent=1, sort_keys=True), encoding="utf-8")
    return manifest


def load_manifest(root: Path | str, expected_shape: tuple[int, int] | None = None) -> dict:
    """The validated manifest of an artefact; ``expected_shape`` = (hidden, intermediate) to enforce."""
    path = Path(root) / MANIFEST_FILE
    if not path.is_file():
        raise FileNotFoundError(f"Missing packed-record manifest: {path}")
    manifest = json.loads(path.read_text(encoding="utf-8"))
    if manifest.get("format") != FORMAT or manifest.get("format_version") != FORMAT_VERSION:
        raise ValueError(f"Unsupported packed-record format: {manifest.get('format')!r} "
                         f"version {manifest.get('format_version')!r}")
    for field in ("dtype", "hidden", "hidden_pad", "intermediate", "record_bytes", "records", "record_offset",
                  "total_intermediate"):
        if field not in manifest:
            raise ValueError(f"Manifest missing required field: {field}")
    if manifest["dtype"] not in _DTYPES:
        raise ValueError(f"Unsupported record dtype {manifest['dtype']!r}")
    hidden, hp, n = manifest["hidden"], manifest["hidden_pad"], manifest["intermediate"]
    esize = torch.empty((), dtype=_DTYPES[manifest["dtype"]]).element_size()
    if hidden < 1 or hp != (hidden + 7) // 8 * 8 or manifest["record_bytes"] != 3 * hp * esize or n < 0:
        raise ValueError("Manifest shape fields are inconsistent")
    record = manifest["records"]
    if not isinstance(record, dict) or {"file", "file_bytes", "sha256"} - set(record):
        raise ValueError("Manifest records entry must give file, file_bytes and sha256")
    if record["file_bytes"] != n * manifest["record_bytes"]:
        raise ValueError("Manifest records byte size does not match intermediate x record_bytes")
    if expected_shape is not None and (hidden, n) != tuple(expected_shape):
        raise ValueError(f"Packed records are {(hidden, n)}, expected {tuple(expected_shape)}")
    return manifest


def validate_files(root: Path | str, manifest: dict, checksums: bool = True) -> None:
    """Payload present, of the recorded size and (optionally) digest."""
    record = manifest["records"]
    path = Path(root) / record["file"]
    if not path.is_file():
        raise FileNotFoundError(f"Missing packed-record payload: {path}")
    if path.stat().st_size != record["file_bytes"]:
        raise ValueError(f"Packed-record byte-size mismatch: {path}")
    if checksums and file_sha256(path) != record["sha256"]:
        raise ValueError(f"Packed-record checksum mismatch: {path}")


def read_records(root: Path | str, manifest: dict | None = None, record_range: tuple[int, int] | None = None,
                 pin: bool = False) -> torch.Tensor:
    """Host tensor ``[rows, 3 * Hp]`` of the records in ``record_range`` (all by default).

    Reads only those rows from disk; ``pin=True`` returns page-locked memory
    (what the host-offload store reads over PCIe).
    """
    manifest = manifest if manifest is not None else load_manifest(root)
    n, width = manifest["intermediate"], 3 * manifest["hidden_pad"]
    dtype = _DTYPES[manifest["dtype"]]
    begin, end = record_range if record_range is not None else (0, n)
    if not 0 <= begin <= end <= n:
        raise ValueError(f"record range {record_range} outside [0, {n}]")
    rb = manifest["record_bytes"]
    out = torch.empty((end - begin, width), dtype=dtype, pin_memory=pin)
    if end > begin:
        view = memoryview(out.view(torch.uint8).view(-1).numpy())
        with (Path(root) / manifest["records"]["file"]).open("rb") as handle:
            handle.seek(begin * rb)
            got = 0
            while got < len(view):
                n_read = handle.readinto(view[got:])
                if not n_read:
                    raise ValueError("Packed-record payload ended early")
                got += n_read
    return out


def load_packed_layer(root: Path | str, device: torch.device | str = "cuda", *,
                      record_range: tuple[int, int] | None = None, checksums: bool = True,
                      expected_shape: tuple[int, int] | None = None) -> PackedFFNWeights:
    """The artefact's layer (or the contiguous shard ``record_range``) as ``PackedFFNWeights`` on ``device``."""
    manifest = load_manifest(root, expected_shape)
    validate_files(root, manifest, checksums)
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("packed layers live on a CUDA device (no CPU fallback)")
    n = manifest["intermediate"]
    begin, end = record_range if record_range is not None else (0, n)
    host = read_records(root, manifest, (begin, end), pin=True)
    packed = host.to(device, non_blocking=True)
    torch.cuda.current_stream(device).synchronize()
    return PackedFFNWeights(packed, manifest["hidden"], end - begin, manifest["record_offset"] + begin,
                            manifest["total_intermediate"])


def pack_safetensors_layer(source: Path | str, output: Path | str) -> dict:
    """Pack a reference runtime-weights file (gate / up / down_proj.weight) into an artefact.

    The counterpart of reference runtime/weights.py:89-96 for the interleaved
    layout; the source's safetensors metadata is carried over.
    """
    from safetensors import safe_open
    from safetensors.torch import load_file

    source = Path(source)
    weights = load_file(str(source), device="cpu")
    missing = [role for role in ROLES if role not in weights]
    if missing:
        raise ValueError(f"runtime weights are missing {missing}")
    with safe_open(str(source), framework="pt", device="cpu") as handle:
        metadata = handle.metadata() or {}
    gate, up, down = (weights[role] for role in ROLES)
    packed = pack_records_host(gate, up, down)
    meta = dict(metadata)
    meta.update(runtime_layout="neuron_major_interleaved", source_artifact=str(source))
    return write_artefact(output, PackedFFNWeights(packed, gate.shape[1], gate.shape[0]), source=str(source),
                          metadata=meta)
