"""Expert bank: the on-disk format the slot refills read from.

Same layout as preemptLM's bank (preempt/datamodel/expert_bank/): a directory
with ``experts.bin`` and ``manifest.json``.  The blob of expert (block b,
expert e) sits at ``(b * num_routed_experts + e) * aligned_blob_size``
(writer.py:90-130), zero-padded to the alignment (4096 by default), and holds
the expert's tensors concatenated in ``tensor_specs`` order (gate, up, down x
weight[, scales, biases]; blob.py:13-69).  The manifest JSON keys are those of
``ExpertBankManifest`` (manifest.py:46-102), so banks written by either side
read on the other.

``PreadExpertBank`` reads a blob with one positioned read straight into a
(pinned, when CUDA is present) host buffer, ready for ``cudaMemcpyAsync``.
"""

from __future__ import annotations

import json
import os
import re
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np
import torch

EXPERT_BANK_SCHEMA_VERSION = 1
MANIFEST_FILENAME = "manifest.json"
EXPERTS_FILENAME = "experts.bin"

# encoding tags (core/constants.py:39-45, encoding.py:19-120)
BACKENDS = frozenset({"mlx"})
KNOWN_DTYPES = frozenset({"int8", "int16", "int32", "uint8", "uint16", "uint32", "bfloat16", "float16", "float32"})
QUANTIZED_REGEX = re.compile(
    r"^(?P<backend>[a-z0-9]+)-(?P<mode>[a-z0-9_]+)-q(?P<bits>\d+)-g(?P<group_size>\d+)-(?P<dtype>[a-z0-9]+)$")
UNQUANTIZED_REGEX = re.compile(r"^(?P<backend>[a-z0-9]+)-unquantized-(?P<dtype>[a-z0-9]+)$")
_TAG_GRAMMAR = ("<backend>-<mode>-q<bits>-g<group_size>-<scalar>", "<backend>-unquantized-<scalar>")


class ReadPriority:
    """Lower is more urgent (core/enums.py:20-28)."""

    DEMAND = 0
    PREFETCH = 1


@dataclass(frozen=True)
class ExpertBankEncoding:
    backend: str
    mode: str | None
    bits: int | None
    group_size: int | None
    dtype: str

    @property
    def is_quantized(self) -> bool:
        return self.mode is not None

    @classmethod
    def from_tag(cls, tag: str) -> "ExpertBankEncoding":
        return parse_encoding_tag(tag)


def parse_encoding_tag(tag: str) -> ExpertBankEncoding:
    """Decode ``mlx-affine-q4-g64-bfloat16`` / ``mlx-unquantized-bfloat16``
    (encoding.py:61-120); raises ValueError with the same wording classes."""
    m = UNQUANTIZED_REGEX.match(tag) or QUANTIZED_REGEX.match(tag)
    if m is None:
        raise ValueError(f"Malformed encoding tag {tag!r}. Valid formats: {', '.join(_TAG_GRAMMAR)!r}")
    backend = m["backend"]
    if backend not in BACKENDS:
        raise ValueError(f"Unknown encoding backend {backend!r} in tag {tag!r}; known families: {sorted(BACKENDS)!r}.")
    scalar = m["dtype"]
    if scalar not in KNOWN_DTYPES:
        raise ValueError(f"Unknown encoding scalar {scalar!r} in tag {tag!r}; known scalars: {sorted(KNOWN_DTYPES)!r}.")
    g = m.groupdict()
    if "bits" not in g:
        return ExpertBankEncoding(backend, None, None, None, scalar)
    bits, gs = int(g["bits"]), int(g["group_size"])
    if bits < 1 or gs < 1:
        raise ValueError(f"Malformed encoding tag {tag!r}: bits and group size must be positive, "
                         f"but got bits={bits!r} and group_size={gs!r}.")
    return ExpertBankEncoding(backend, g["mode"], bits, gs, scalar)


def make_encoding_tag(bits: int | None, group_size: int | None = 64, dtype: str = "bfloat16",
                      mode: str = "affine") -> str:
    if bits is None:
        return f"mlx-unquantized-{dtype}"
    return f"mlx-{mode}-q{bits}-g{group_size}-{dtype}"


@dataclass(frozen=True)
class TensorSpec:
    """identity.py:32-53."""

    name: str
    dtype: str
    shape: tuple[int, ...]
    num_bytes: int

    def to_json(self) -> dict:
        return {"name": self.name, "dtype": self.dtype, "shape": list(self.shape), "num_bytes": self.num_bytes}


@dataclass(frozen=True)
class ModelMoESpec:
    moe_block_idxs: tuple[int, ...]
    num_routed_experts: int
    top_k: int

    @property
    def total_routed_experts(self) -> int:
        return len(self.moe_block_idxs) * self.num_routed_experts


@dataclass(frozen=True)
class ExpertBlobDescriptor:
    offset: int
    length: int
    block_idx: int
    expert_idx: int


@dataclass(frozen=True)
class ExpertBankManifest:
    model_id: str
    model_fingerprint: str
    encoding: str
    tensor_specs: tuple[TensorSpec, ...]
    model_moe_spec: ModelMoESpec
    blob_index: tuple[ExpertBlobDescriptor, ...]
    alignment: int = 4096
    schema_version: int = EXPERT_BANK_SCHEMA_VERSION

    def __post_init__(self):  # manifest.py:72-98
        if len(self.blob_index) != self.model_moe_spec.total_routed_experts:
            raise ValueError("blob index size does not match the MoE topology")
        expected = self.expert_num_bytes()
        seen, offsets = set(), set()
        for b in self.blob_index:
            if b.length != expected:
                raise ValueError(f"blob ({b.block_idx}, {b.expert_idx}) is {b.length} bytes, expected {expected}")
            if (b.block_idx, b.expert_idx) in seen:
                raise ValueError("Manifest contains duplicate blobs")
            if b.offset in offsets:
                raise ValueError("Manifest contains duplicate blob offsets")
            seen.add((b.block_idx, b.expert_idx))
            offsets.add(b.offset)

    def expert_num_bytes(self) -> int:
        return sum(s.num_bytes for s in self.tensor_specs)

    def to_json(self) -> dict:
        return {
            "schema_version": self.schema_version, "model_id": self.model_id,
            "model_fingerprint": self.model_fingerprint, "encoding": self.encoding,
            "tensor_specs": [s.to_json() for s in self.tensor_specs],
            "model_moe_spec": {"moe_block_idxs": list(self.model_moe_spec.moe_block_idxs),
                               "num_routed_experts": self.model_moe_spec.num_routed_experts,
                               "top_k": self.model_moe_spec.top_k},
            "alignment": self.alignment,
            "blob_index": [{"offset": b.offset, "length": b.length, "block_idx": b.block_idx,
                            "expert_idx": b.expert_idx} for b in self.blob_index],
        }

    def save(self, path: Path) -> Path:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        out = path / MANIFEST_FILENAME
        out.write_text(json.dumps(self.to_json(), indent=2), encoding="utf-8")
        return out

    @classmethod
    def load(cls, path: Path) -> "ExpertBankManifest":
        raw = json.loads((Path(path) / MANIFEST_FILENAME).read_text(encoding="utf-8"))
        return cls(
            model_id=raw["model_id"], model_fingerprint=raw["model_fingerprint"], encoding=raw["encoding"],
            tensor_specs=tuple(TensorSpec(s["name"], s["dtype"], tuple(s["shape"]), s["num_bytes"])
                               for s in raw["tensor_specs"]),
            model_moe_spec=ModelMoESpec(tuple(raw["model_moe_spec"]["moe_block_idxs"]),
                                        raw["model_moe_spec"]["num_routed_experts"], raw["model_moe_spec"]["top_k"]),
            blob_index=tuple(ExpertBlobDescriptor(b["offset"], b["length"], b["block_idx"], b["expert_idx"])
                             for b in raw["blob_index"]),
            alignment=raw.get("alignment", 4096), schema_version=raw.get("schema_version", 1),
        )


@dataclass(frozen=True)
class SerializedExpert:
    """One expert's bytes plus the specs that decode them (blob.py:13-34).
    ``data`` is a host uint8 tensor (pinned when read for a GPU) or bytes."""

    idx: int
    data: object
    encoding: str
    tensor_specs: tuple[TensorSpec, ...]

    def as_tensor(self) -> torch.Tensor:
        if isinstance(self.data, torch.Tensor):
            return self.data
        return torch.frombuffer(bytearray(self.data), dtype=torch.uint8)

    def nbytes(self) -> int:
        return int(self.data.numel()) if isinstance(self.data, torch.Tensor) else len(self.data)


_NP_DTYPES = {"bfloat16": np.uint16}


def decode_serialized_expert(expert: SerializedExpert, encoding: ExpertBankEncoding | None = None) -> dict:
    """Split a blob into named numpy arrays in spec order (expert_cache.py:24-80).
    bf16 tensors come back as uint16 bit patterns."""
    if encoding is not None and (parsed := parse_encoding_tag(expert.encoding)) != encoding:
        raise ValueError(f"Encoding mismatch for {expert.idx}. Expected {encoding!r}, but got "
                         f"{expert.encoding!r} ({parsed!r}).")
    buf = expert.as_tensor().numpy().tobytes() if isinstance(expert.data, torch.Tensor) else bytes(expert.data)
    out, off = {}, 0
    for s in expert.tensor_specs:
        dt = np.dtype(_NP_DTYPES.get(s.dtype, s.dtype))
        count = int(np.prod(s.shape))
        out[s.name] = np.frombuffer(buf, dtype=dt, count=count, offset=off).reshape(s.shape)
        off += count * dt.itemsize
    if off != len(buf):
        raise ValueError(f"Blob for {expert.idx} is {len(buf)} bytes, but its tensor spec accounts for {off} bytes.")
    return out


def derive_tensor_specs(arrays, order) -> tuple[TensorSpec, ...]:
    return tuple(TensorSpec(n, _dtype_name(arrays[n]), tuple(arrays[n].shape), _nbytes(arrays[n])) for n in order)


def _dtype_name(a) -> str:
    if isinstance(a, torch.Tensor):
        return {torch.bfloat16: "bfloat16", torch.int32: "uint32", torch.uint8: "uint8"}.get(a.dtype, str(a.dtype))
    return str(a.dtype)


def _nbytes(a) -> int:
    return a.numel() * a.element_size() if isinstance(a, torch.Tensor) else a.nbytes


def assemble_expert_blob(arrays, specs) -> bytes:
    parts = []
    for s in specs:
        a = arrays[s.name]
        if _dtype_name(a) != s.dtype and not isinstance(a, torch.Tensor):
            raise ValueError(f"Tensor {s.name!r}: dtype {a.dtype} != spec {s.dtype}.")
        if tuple(a.shape) != tuple(s.shape):
            raise ValueError(f"Tensor {s.name!r}: shape {tuple(a.shape)} != spec {s.shape}.")
        if isinstance(a, torch.Tensor):
            a = a.detach().cpu().contiguous().view(torch.uint8).numpy()
        parts.append(np.ascontiguousarray(a).tobytes())
    return b"".join(parts)


class ExpertBankWriter:
    """writer.py:28-169: blob (b, e) at (b*E + e) * aligned_size, zero padded."""

    def __init__(self, expert_bank_path, *, model_id: str, model_fingerprint: str, encoding: str,
                 tensor_specs: tuple[TensorSpec, ...], model_moe_spec: ModelMoESpec, alignment: int = 4096,
                 overwrite: bool = False):
        self.path = Path(expert_bank_path)
        self.model_id, self.model_fingerprint, self.encoding = model_id, model_fingerprint, encoding
        self.tensor_specs, self.model_moe_spec, self._alignment = tensor_specs, model_moe_spec, alignment
        self._blob_size = sum(s.num_bytes for s in tensor_specs)
        self._aligned = (self._blob_size + alignment - 1) // alignment * alignment
        self._blobs: list[ExpertBlobDescriptor | None] = [None] * model_moe_spec.total_routed_experts
        self._num_writes = 0
        self._is_closed = False
        bin_path = self.path / EXPERTS_FILENAME
        if bin_path.exists() and not overwrite:
            raise FileExistsError(f"Expert bank already exists at {self.path.as_posix()!r}.")
        self.path.mkdir(parents=True, exist_ok=True)
        (self.path / MANIFEST_FILENAME).unlink(missing_ok=True)
        self._file = bin_path.open("wb")

    @property
    def aligned_blob_size(self) -> int:
        return self._aligned

    def add_expert(self, block_idx: int, expert_idx: int, data: bytes) -> None:
        if len(data) != self._blob_size:
            raise ValueError(f"expert blob must be {self._blob_size} bytes, got {len(data)}")
        pos = self.model_moe_spec.moe_block_idxs.index(block_idx) if block_idx in self.model_moe_spec.moe_block_idxs \
            else None
        if pos is None:
            raise ValueError(f"block {block_idx} is not a MoE block of this bank")
        # writer.py:97-98 indexes by the transformer block id; blobs of a
        # contiguous MoE block list land at the same offsets either way.
        glob = block_idx * self.model_moe_spec.num_routed_experts + expert_idx
        slot = pos * self.model_moe_spec.num_routed_experts + expert_idx
        if self._blobs[slot] is not None:
            raise ValueError(f"Duplicate expert ({block_idx}, {expert_idx})")
        off = glob * self._aligned
        self._file.seek(off)
        self._file.write(data)
        pad = self._aligned - len(data)
        if pad:
            self._file.write(b"\x00" * pad)
        self._blobs[slot] = ExpertBlobDescriptor(off, len(data), block_idx, expert_idx)
        self._num_writes += 1

    def finalize(self) -> ExpertBankManifest:
        if self._is_closed:
            raise RuntimeError("expert bank writer already finalised")
        if self._num_writes != self.model_moe_spec.total_routed_experts:
            raise RuntimeError(f"{self._num_writes} of {self.model_moe_spec.total_routed_experts} experts written")
        self._file.close()
        self._is_closed = True
        m = ExpertBankManifest(self.model_id, self.model_fingerprint, self.encoding, self.tensor_specs,
                               self.model_moe_spec, tuple(self._blobs), alignment=self._alignment)
        m.save(self.path)
        return m

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        if exc_type is not None:
            self._file.close()
            return
        if not self._is_closed:
            self.finalize()


def _host_buffer(nbytes: int, pinned: bool) -> torch.Tensor:
    return torch.empty(nbytes, dtype=torch.uint8, pin_memory=pinned)


DIRECT_IO_ALIGN = 4096  # file offset, length and buffer alignment of an O_DIRECT read


class PreadExpertBank:
    """banks.py:130-206: positioned reads of ``experts.bin``.  ``read_sync``
    fills a fresh host buffer; ``read_into`` fills a caller buffer.

    With ``bypass_page_cache`` (the reference opens the file F_NOCACHE on
    darwin, banks.py:140-148) blobs are read with O_DIRECT where the file
    system supports it: the blob offsets are 4096-aligned (writer.py:90-95),
    the read length is rounded up to 4096 within the blob's zero padding and
    the destination is a 4096-aligned slice of the host buffer, so the read
    goes straight from the device into (pinned) memory.  Where O_DIRECT is
    refused (tmpfs, for one) the read is buffered and its pages are dropped
    from the page cache right after it, so a later miss on the same blob reads
    the disk again instead of the page cache."""

    def __init__(self, expert_bank_path, bypass_page_cache: bool = False, pinned: bool | None = None):
        self.path = Path(expert_bank_path)
        self._manifest = ExpertBankManifest.load(self.path)
        self._tensor_specs = self._manifest.tensor_specs
        self._pinned = torch.cuda.is_available() if pinned is None else pinned
        self._fd: int | None = os.open(self.path / EXPERTS_FILENAME, os.O_RDONLY)
        self._dfd: int | None = None
        self._drop_pages = False
        if bypass_page_cache:
            if hasattr(os, "O_DIRECT") and self._manifest.alignment % DIRECT_IO_ALIGN == 0:
                try:
                    self._dfd = os.open(self.path / EXPERTS_FILENAME, os.O_RDONLY | os.O_DIRECT)
                except OSError:
                    self._dfd = None
            self._drop_pages = self._dfd is None and hasattr(os, "posix_fadvise")
            if hasattr(os, "posix_fadvise"):
                os.posix_fadvise(self._fd, 0, 0, os.POSIX_FADV_DONTNEED)

    @property
    def direct_io(self) -> bool:
        """Whether blob reads bypass the page cache by O_DIRECT."""
        return self._dfd is not None

    @property
    def manifest(self) -> ExpertBankManifest:
        return self._manifest

    @property
    def blob_index(self) -> tuple[ExpertBlobDescriptor, ...]:
        return self._manifest.blob_index

    @property
    def model_fingerprint(self) -> str:
        return self._manifest.model_fingerprint

    def _validate_fd(self) -> int:
        if self._fd is None:
            raise RuntimeError("Cannot read closed expert bank.")
        return self._fd

    def _direct_span(self, blob) -> int:
        """Bytes an O_DIRECT read of ``blob`` covers (0: read it buffered)."""
        if self._dfd is None or blob.offset % DIRECT_IO_ALIGN:
            return 0
        return (blob.length + DIRECT_IO_ALIGN - 1) // DIRECT_IO_ALIGN * DIRECT_IO_ALIGN

    def read_into(self, expert_idx: int, buf: torch.Tensor) -> SerializedExpert:
        fd = self._validate_fd()
        if not 0 <= expert_idx < len(self.blob_index):
            raise KeyError(expert_idx)
        blob = self.blob_index[expert_idx]
        span = self._direct_span(blob)
        if span and buf.numel() >= span and buf.data_ptr() % DIRECT_IO_ALIGN == 0:
            view = memoryview(buf.numpy()).cast("B")[:span]
            try:
                got = os.preadv(self._dfd, [view], blob.offset)  # may stop at end of file inside the padding
            except OSError:  # the device refused this direct read: read it buffered
                got = -1
            if got >= blob.length:
                return SerializedExpert(expert_idx, buf[: blob.length], self._manifest.encoding, self._tensor_specs)
        view = memoryview(buf.numpy()).cast("B")[: blob.length]
        got = os.preadv(fd, [view], blob.offset)
        if got != blob.length:
            raise IOError(f"short read of expert {expert_idx}: {got} of {blob.length} bytes")
        if self._drop_pages:
            os.posix_fadvise(fd, blob.offset, blob.length, os.POSIX_FADV_DONTNEED)
        return SerializedExpert(expert_idx, buf[: blob.length], self._manifest.encoding, self._tensor_specs)

    def read_sync(self, expert_idx: int, priority: int = ReadPriority.DEMAND) -> SerializedExpert:
        if not 0 <= expert_idx < len(self.blob_index):
            raise KeyError(expert_idx)
        blob = self.blob_index[expert_idx]
        span = self._direct_span(blob)
        if span:  # a 4096-aligned slice of a slightly larger buffer
            raw = _host_buffer(span + DIRECT_IO_ALIGN, self._pinned)
            off = (-raw.data_ptr()) % DIRECT_IO_ALIGN
            return self.read_into(expert_idx, raw[off: off + span])
        return self.read_into(expert_idx, _host_buffer(blob.length, self._pinned))

    def check_model_compatibility(self, model_id: str, num_routed_experts: int, top_k: int,
                                  moe_block_idxs: tuple[int, ...]) -> None:
        m = self._manifest
        exp = {"model_id": m.model_id, "num_routed_experts": m.model_moe_spec.num_routed_experts,
               "top_k": m.model_moe_spec.top_k, "moe_block_idxs": tuple(m.model_moe_spec.moe_block_idxs)}
        obs = {"model_id": model_id, "num_routed_experts": num_routed_experts, "top_k": top_k,
               "moe_block_idxs": tuple(moe_block_idxs)}
        bad = {k: (exp[k], obs[k]) for k in exp if exp[k] != obs[k]}
        if bad:
            raise ValueError(f"expert bank incompatible with model: {bad!r}")

    def close(self) -> None:
        if self._dfd is not None:
            os.close(self._dfd)
            self._dfd = None
        if self._fd is not None:
            os.close(self._fd)
            self._fd = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
