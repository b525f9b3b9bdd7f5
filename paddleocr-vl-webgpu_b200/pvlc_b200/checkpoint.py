"""PaddleOCR-VL-1.6 checkpoint import: a BF16 safetensors file into the engine's fp16 weights.

Host side (no GPU needed):
  * ``SafetensorsCatalog`` -- the reference's bounded, header-only safetensors importer
    (crates/pvlc-safetensors/src/lib.rs:1-803): opening reads the 8-byte prefix and the
    JSON header only, validates every declared tensor and the payload layout, and
    reports the reference's ``ImportErrorCode`` names in the reference's precedence;
    payloads are copied later in bounded chunks.
  * ``schema_specs`` / ``validate_schema`` -- the exact tensor catalog of the one
    supported checkpoint and its validator (crates/pvlc-model-schema/src/lib.rs:140-495),
    parameterised by ``ModelConfig`` so that the default configuration yields exactly
    the reference's 620 tensors (pinned by the catalog digests of
    crates/pvlc-model-schema/tests/schema_contract.rs:8-13).
  * ``fp16_output_header`` -- the self-describing header of the reference's FP16
    checkpoint (crates/pvlc-safetensors/src/fp16.rs:403-437).

Device side: the BF16 payload is read in bounded chunks into pinned host buffers, copied
to HBM and converted in place by the library's ``pvlc_bf16_to_f16`` kernel (the
reference's ``finite_bf16_to_f16_bits`` rule, fp16.rs:171-210), which also reports the
first rejected element (NaN / infinity, or beyond the f16 range) the way the reference's
stream converter does (fp16.rs:212-276).  ``load_weights`` turns the converted payload
into the engine's weight lists without a host-side FP16 file;
``convert_bf16_checkpoint_to_f16`` writes the reference's FP16 file (same header, same
payload bits) with the conversion on the GPU.  There is no CPU conversion path: the
device kernel is the product, and a missing CUDA library raises.
"""
from __future__ import annotations

import json
import os
import stat
import struct
from dataclasses import dataclass, field

import numpy as np

MAX_HEADER_BYTES = 100_000_000          # crates/pvlc-safetensors/src/lib.rs:25
COPY_BUFFER_BYTES = 64 * 1024           # lib.rs:26 (the host-side copy chunk)
FP16_CHECKPOINT_CONVERSION_ID = "bf16_to_ieee_f16_rne_v1"   # fp16.rs:14
MODEL_ID = "PaddlePaddle/PaddleOCR-VL-1.6"                  # pvlc-model-schema/src/lib.rs:10
MODEL_REVISION = "66317acc4c9fc17bd154591ce650735cd2855f3e"
PACKING_POSITIONS = 32_768              # packing_position_embedding rows (lib.rs:358-363)
DEVICE_CHUNK_BYTES = 64 << 20           # payload bytes per device conversion launch

# dtype name -> byte width (pvlc-model-schema/src/lib.rs:34-70)
DTYPE_BYTES = {"BOOL": 1, "U8": 1, "I8": 1, "F8_E4M3": 1, "F8_E5M2": 1, "U16": 2, "I16": 2,
               "BF16": 2, "F16": 2, "U32": 4, "I32": 4, "F32": 4, "U64": 8, "I64": 8, "F64": 8}
_U64_MAX = (1 << 64) - 1


class SafetensorsImportError(Exception):
    """The reference's ``ImportError`` (lib.rs:71-151): ``code`` is an ``ImportErrorCode``
    name (lib.rs:46-69), ``tensor_name`` the tensor it concerns, if any."""

    def __init__(self, code: str, message: str, tensor_name: str | None = None):
        self.code = code
        self.tensor_name = tensor_name
        text = f"safetensors import error {code}: {message}"
        if tensor_name is not None:
            text += f" (tensor {tensor_name!r})"
        super().__init__(text)


def _fail(code: str, message: str, tensor_name: str | None = None):
    return SafetensorsImportError(code, message, tensor_name)


class SchemaError(Exception):
    """pvlc-model-schema/src/lib.rs:96-138: ``code`` is one of DuplicateTensor,
    UnexpectedTensor, DtypeMismatch, ShapeMismatch, MissingTensor."""

    def __init__(self, code: str, tensor_name: str):
        self.code = code
        self.tensor_name = tensor_name
        super().__init__(f"checkpoint schema error {code} for tensor {tensor_name!r}")


class Fp16CheckpointError(Exception):
    """fp16.rs:16-150: ``code`` is one of Io, InvalidSource, UnsupportedSourceDtype,
    NonFiniteSource, OutOfRangeSource, SourceChanged, SourceDestinationAlias,
    OutputAlreadyExists; ``element_index`` is the rejected element within its tensor."""

    def __init__(self, code: str, message: str, tensor_name: str | None = None,
                 element_index: int | None = None):
        self.code = code
        self.tensor_name = tensor_name
        self.element_index = element_index
        text = f"FP16 checkpoint conversion error {code}: {message}"
        if tensor_name is not None:
            text += f" (tensor {tensor_name!r}"
            if element_index is not None:
                text += f", element {element_index}"
            text += ")"
        super().__init__(text)


# ----------------------------------------------------------------------------- catalog
@dataclass(frozen=True)
class TensorHeader:
    name: str
    dtype: str
    shape: tuple
    data_offsets: tuple   # relative to the start of the data section

    @property
    def byte_len(self) -> int:
        return self.data_offsets[1] - self.data_offsets[0]


class _Obj(list):
    """A JSON object as its (key, value) pairs in document order, duplicates kept."""


def _reject_constant(name):
    raise ValueError(f"invalid JSON literal {name}")


def _has_surrogate(s: str) -> bool:
    return any(0xD800 <= ord(c) <= 0xDFFF for c in s)


def _u64_list(value, field_name):
    if not isinstance(value, list):
        raise _fail("InvalidTensorMetadata", f"{field_name} must be an array")
    for v in value:
        if isinstance(v, bool) or not isinstance(v, int) or v < 0 or v > _U64_MAX:
            raise _fail("InvalidTensorMetadata", f"{field_name} must contain unsigned integers")
    return value


def _parse_header(text: str):
    """Walks the header in document order with the checks of the reference's serde
    visitors (lib.rs:645-803): duplicate keys at any level it reads, string-only
    metadata, exactly dtype / shape / data_offsets per tensor."""
    try:
        root = json.loads(text, object_pairs_hook=_Obj, parse_constant=_reject_constant)
    except ValueError as e:   # json.JSONDecodeError is a ValueError
        raise _fail("InvalidHeaderJson", str(e)) from None
    if not isinstance(root, _Obj):
        raise _fail("InvalidHeaderJson", "expected a safetensors header object")
    seen, metadata, tensors = set(), {}, []
    for key, value in root:
        if _has_surrogate(key):
            raise _fail("InvalidHeaderJson", "lone surrogate in a key")
        if key in seen:
            raise _fail("DuplicateHeaderKey", key)
        seen.add(key)
        if key == "__metadata__":
            if not isinstance(value, _Obj):
                raise _fail("InvalidHeaderJson", "metadata must be an object")
            for mk, mv in value:
                if mk in metadata:
                    raise _fail("DuplicateHeaderKey", f"metadata.{mk}")
                if not isinstance(mv, str):
                    raise _fail("InvalidMetadata", f"metadata.{mk} is not a string")
                if _has_surrogate(mk) or _has_surrogate(mv):
                    raise _fail("InvalidHeaderJson", "lone surrogate in metadata")
                metadata[mk] = mv
            continue
        if not isinstance(value, _Obj):
            raise _fail("InvalidHeaderJson", f"tensor {key!r} is not an object")
        fields = {}
        for fk, fv in value:
            if fk in fields:
                raise _fail("DuplicateHeaderKey", f"tensor field {fk}")
            if fk not in ("dtype", "shape", "data_offsets"):
                raise _fail("InvalidTensorMetadata", f"unknown field {fk}")
            fields[fk] = fv
        if "dtype" not in fields:
            raise _fail("InvalidTensorMetadata", "missing dtype")
        if not isinstance(fields["dtype"], str):
            raise _fail("InvalidTensorMetadata", "dtype has the wrong type")
        shape = _u64_list(fields.get("shape"), "shape")
        offsets = _u64_list(fields.get("data_offsets"), "data_offsets")
        if len(offsets) != 2:
            raise _fail("InvalidTensorMetadata", "data_offsets must contain two integers")
        tensors.append((key, fields["dtype"], shape, offsets))
    return metadata, tensors


def _validate_tensor(name, dtype, shape, offsets) -> TensorHeader:
    """lib.rs:514-571 (validate_tensor)."""
    if not name:
        raise _fail("InvalidTensorMetadata", "tensor name is empty", name)
    if dtype not in DTYPE_BYTES:
        raise _fail("UnsupportedDtype", f"unsupported dtype {dtype!r}", name)
    count = 1
    for d in shape:
        count *= d
        if count > _U64_MAX:
            raise _fail("ShapeElementCountOverflow", "shape element count overflows u64", name)
    expected = count * DTYPE_BYTES[dtype]
    if expected > _U64_MAX:
        raise _fail("ShapeElementCountOverflow", "tensor byte count overflows u64", name)
    start, end = offsets
    if end < start:
        raise _fail("InvalidDataOffsets", "tensor data offsets are reversed", name)
    if end - start != expected:
        raise _fail("TensorByteLengthMismatch",
                    f"shape requires {expected} bytes but offsets span {end - start}", name)
    return TensorHeader(name, dtype, tuple(shape), (start, end))


def _validate_layout(tensors, body_len):
    """lib.rs:573-607: payloads tile the data section exactly, in offset order."""
    cursor = 0
    for t in sorted(tensors, key=lambda t: (t.data_offsets[0], t.data_offsets[1],
                                            t.name.encode())):
        if t.data_offsets[0] < cursor:
            raise _fail("OverlappingData", "tensor payload overlaps a previous tensor", t.name)
        if t.data_offsets[0] > cursor:
            raise _fail("NonContiguousData", "tensor payload leaves an unclaimed gap", t.name)
        cursor = t.data_offsets[1]
    if cursor != body_len:
        raise _fail("DataLengthMismatch",
                    f"tensor data covers {cursor} bytes but file body is {body_len} bytes")


def _open_regular_file(path):
    """lib.rs:440-476: only a regular file (not a symlink), unchanged while opening."""
    try:
        before = os.lstat(path)
    except OSError as e:
        raise _fail("Io", f"cannot inspect {path}: {e}") from e
    if not stat.S_ISREG(before.st_mode):
        raise _fail("NotRegularFile", f"{path} is not a regular file")
    try:
        fh = open(path, "rb")
    except OSError as e:
        raise _fail("Io", f"cannot open {path}: {e}") from e
    after = os.fstat(fh.fileno())
    if not stat.S_ISREG(after.st_mode) or (before.st_dev, before.st_ino) != \
            (after.st_dev, after.st_ino):
        fh.close()
        raise _fail("NotRegularFile", f"{path} changed while it was being opened")
    return fh, after.st_size


def _read_exact(fh, n, truncated_code):
    try:
        data = fh.read(n)
    except OSError as e:
        raise _fail("Io", f"failed to read safetensors header: {e}") from e
    if len(data) != n:
        raise _fail(truncated_code, "safetensors header is truncated")
    return data


@dataclass
class SafetensorsCatalog:
    """crates/pvlc-safetensors/src/lib.rs:153-437 (SafetensorsCatalog)."""
    file_len: int
    header_len: int
    data_start: int
    tensors: list                       # TensorHeader, sorted by name (bytewise)
    metadata: dict
    source_path: str | None = None
    _index: dict = field(default_factory=dict, repr=False)

    @classmethod
    def open(cls, path) -> "SafetensorsCatalog":
        path = os.fspath(path)
        fh, file_len = _open_regular_file(path)
        with fh:
            cat = cls.read_from(fh, file_len)
        cat.source_path = path
        return cat

    @classmethod
    def read_from(cls, reader, file_len: int) -> "SafetensorsCatalog":
        """Parses only the prefix and the header from a reader at byte zero
        (lib.rs:193-243); file_len bounds every declared offset."""
        if file_len < 8:
            raise _fail("HeaderPrefixTruncated",
                        "file is shorter than the eight-byte header prefix")
        header_len = struct.unpack("<Q", _read_exact(reader, 8, "HeaderPrefixTruncated"))[0]
        if header_len > MAX_HEADER_BYTES:
            raise _fail("HeaderTooLarge", f"declared header is {header_len} bytes")
        if header_len % 8:
            raise _fail("HeaderLengthNotAligned",
                        f"declared header length {header_len} is not eight-byte aligned")
        data_start = 8 + header_len
        if data_start > file_len:
            raise _fail("HeaderTruncated", "declared header extends beyond the file")
        raw = _read_exact(reader, header_len, "HeaderTruncated")
        try:
            text = raw.decode("utf-8")
        except UnicodeDecodeError as e:
            raise _fail("InvalidHeaderUtf8", f"header is not UTF-8: {e}") from None
        metadata, raw_tensors = _parse_header(text)
        tensors = [_validate_tensor(*t) for t in raw_tensors]
        _validate_layout(tensors, file_len - data_start)
        tensors.sort(key=lambda t: t.name.encode())
        cat = cls(file_len, header_len, data_start, tensors, dict(sorted(metadata.items())))
        cat._index = {t.name: t for t in tensors}
        return cat

    @property
    def body_len(self) -> int:
        return self.file_len - self.data_start

    def tensor(self, name: str) -> TensorHeader | None:
        return self._index.get(name)

    def _require(self, name: str) -> TensorHeader:
        t = self.tensor(name)
        if t is None:
            raise _fail("TensorNotFound", "tensor is absent from the catalog", name)
        return t

    def validate_paddleocr_vl_16(self, cfg=None) -> None:
        """lib.rs:277-284: the catalog must be exactly the model's tensor catalog."""
        validate_schema([(t.name, t.dtype, t.shape) for t in self.tensors], schema_specs(cfg))

    def copy_tensor_to(self, name: str, writer) -> int:
        """lib.rs:286-300,375-418: the payload of one tensor, 64 KiB at a time."""
        t = self._require(name)
        if self.source_path is None:
            raise _fail("SourceUnavailable", "catalog was created from a borrowed reader")
        fh, file_len = _open_regular_file(self.source_path)
        with fh:
            if file_len != self.file_len:
                raise _fail("DataLengthMismatch", "source file length changed after catalog import")
            fh.seek(self.data_start + t.data_offsets[0])
            remaining, copied = t.byte_len, 0
            while remaining:
                chunk = fh.read(min(remaining, COPY_BUFFER_BYTES))
                if not chunk:
                    raise _fail("Io", "failed to read tensor payload", name)
                writer.write(chunk)
                remaining -= len(chunk)
                copied += len(chunk)
        return copied

    def load_tensor_f32(self, name: str) -> np.ndarray:
        """lib.rs:302-373: BF16 / F16 / F32 payload as f32, every stored bit kept."""
        t = self._require(name)
        if t.dtype not in ("BF16", "F16", "F32"):
            raise _fail("UnsupportedTensorConversion",
                        f"cannot materialize {t.dtype} as f32 values", name)

        class _Sink(bytearray):
            def write(self, b):
                self.extend(b)

        sink = _Sink()
        self.copy_tensor_to(name, sink)
        raw = np.frombuffer(bytes(sink), dtype="<u2" if t.dtype != "F32" else "<u4")
        if t.dtype == "F32":
            return raw.astype(np.uint32).view(np.float32).copy()
        if t.dtype == "BF16":
            return (raw.astype(np.uint32) << 16).view(np.float32)
        return _f16_bits_to_f32(raw)


def _f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    """lib.rs:420-438 (f16_to_f32_bits) in integer arithmetic, NaN payloads kept."""
    h = h.astype(np.uint32)
    sign = (h & 0x8000) << 16
    exp = (h >> 10) & 0x1F
    frac = h & 0x3FF
    bits = sign | ((exp + 112) << 23) | (frac << 13)                 # normal
    bits = np.where(exp == 0x1F, sign | 0x7F800000 | (frac << 13), bits)
    sub = (exp == 0) & (frac != 0)
    sub_vals = (frac.astype(np.float32) * np.float32(2.0 ** -24)).view(np.uint32) | sign
    bits = np.where(sub, sub_vals, bits)
    bits = np.where((exp == 0) & (frac == 0), sign, bits)
    return bits.astype(np.uint32).view(np.float32)


# ------------------------------------------------------------------------------ schema
@dataclass(frozen=True)
class TensorSpec:
    name: str
    dtype: str
    shape: tuple
    semantic_id: str


def schema_specs(cfg=None) -> list:
    """The exact checkpoint catalog (pvlc-model-schema/src/lib.rs:275-495), sorted by
    name.  With the default ModelConfig it is the reference's 620 BF16 tensors; other
    configurations scale the same families (layer counts, widths, vocabulary)."""
    if cfg is None:
        from .model import ModelConfig
        cfg = ModelConfig()
    out = []

    def add(name, shape, semantic):
        out.append(TensorSpec(name, "BF16", tuple(shape), semantic))

    D, V, I = cfg.hidden, cfg.vocab, cfg.intermediate
    VH, VI = cfg.vision_hidden, cfg.vision_intermediate
    M = VH * cfg.merge * cfg.merge
    QW, KW = cfg.query_heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    add("lm_head.weight", [V, D], "lm_head.weight")
    for s in ("bias", "weight"):
        add(f"mlp_AR.pre_norm.{s}", [VH], f"projector.pre_norm.{s}")
        add(f"mlp_AR.linear_1.{s}", [M] if s == "bias" else [M, M], f"projector.linear1.{s}")
        add(f"mlp_AR.linear_2.{s}", [D] if s == "bias" else [D, M], f"projector.linear2.{s}")
    add("model.embed_tokens.weight", [V, D], "decoder.embedding.weight")
    add("model.norm.weight", [D], "decoder.final_norm.weight")
    for layer in range(cfg.decoder_layers):
        p, s = f"model.layers.{layer}", f"decoder.layer.{layer:02d}"
        add(f"{p}.input_layernorm.weight", [D], f"{s}.norm1.weight")
        add(f"{p}.post_attention_layernorm.weight", [D], f"{s}.norm2.weight")
        for proj, sem, shape in (("q_proj", "q", [QW, D]), ("k_proj", "k", [KW, D]),
                                 ("v_proj", "v", [KW, D]), ("o_proj", "out", [D, QW])):
            add(f"{p}.self_attn.{proj}.weight", shape, f"{s}.attention.{sem}.weight")
        for proj, sem, shape in (("gate_proj", "gate", [I, D]), ("up_proj", "up", [I, D]),
                                 ("down_proj", "down", [D, I])):
            add(f"{p}.mlp.{proj}.weight", shape, f"{s}.mlp.{sem}.weight")
    e = "visual.vision_model.embeddings"
    add(f"{e}.packing_position_embedding.weight", [PACKING_POSITIONS, VH],
        "vision.embeddings.packing_position.weight")
    add(f"{e}.patch_embedding.bias", [VH], "vision.embeddings.patch.bias")
    add(f"{e}.patch_embedding.weight", [VH, cfg.channels, cfg.patch_size, cfg.patch_size],
        "vision.embeddings.patch.weight")
    add(f"{e}.position_embedding.weight", [cfg.pos_side * cfg.pos_side, VH],
        "vision.embeddings.position.weight")
    for layer in range(cfg.vision_layers):
        p, s = f"visual.vision_model.encoder.layers.{layer}", f"vision.layer.{layer:02d}"
        for pn, sn in (("layer_norm1", "norm1"), ("layer_norm2", "norm2")):
            for suf in ("bias", "weight"):
                add(f"{p}.{pn}.{suf}", [VH], f"{s}.{sn}.{suf}")
        for proj, bshape, wshape in (("fc1", [VI], [VI, VH]), ("fc2", [VH], [VH, VI])):
            add(f"{p}.mlp.{proj}.bias", bshape, f"{s}.mlp.{proj}.bias")
            add(f"{p}.mlp.{proj}.weight", wshape, f"{s}.mlp.{proj}.weight")
        for pp, sp in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"), ("out_proj", "out")):
            for suf in ("bias", "weight"):
                add(f"{p}.self_attn.{pp}.{suf}", [VH] if suf == "bias" else [VH, VH],
                    f"{s}.attention.{sp}.{suf}")
    h = "visual.vision_model.head"
    for suf in ("bias", "weight"):
        add(f"{h}.attention.in_proj_{suf}", [3 * VH] if suf == "bias" else [3 * VH, VH],
            f"vision.head.attention.qkv.{suf}")
        add(f"{h}.attention.out_proj.{suf}", [VH] if suf == "bias" else [VH, VH],
            f"vision.head.attention.out.{suf}")
        add(f"{h}.layernorm.{suf}", [VH], f"vision.head.norm.{suf}")
        for proj, bshape, wshape in (("fc1", [VI], [VI, VH]), ("fc2", [VH], [VH, VI])):
            add(f"{h}.mlp.{proj}.{suf}", bshape if suf == "bias" else wshape,
                f"vision.head.mlp.{proj}.{suf}")
        add(f"visual.vision_model.post_layernorm.{suf}", [VH], f"vision.post_norm.{suf}")
    add(f"{h}.probe", [1, 1, VH], "vision.head.probe")
    out.sort(key=lambda t: t.name.encode())
    return out


def _compact_json(value) -> bytes:
    return json.dumps(value, separators=(",", ":"), ensure_ascii=False).encode()


def canonical_catalog_bytes(specs) -> bytes:
    """pvlc-model-schema/src/lib.rs:148-168: JSON array of {dtype, name, shape} + LF."""
    return _compact_json([{"dtype": s.dtype, "name": s.name, "shape": list(s.shape)}
                          for s in specs]) + b"\n"


def canonical_semantic_map_bytes(specs) -> bytes:
    """lib.rs:170-190: JSON array of {name, semantic_id} + LF."""
    return _compact_json([{"name": s.name, "semantic_id": s.semantic_id} for s in specs]) + b"\n"


def validate_schema(observed, specs) -> None:
    """lib.rs:192-238: observed (name, dtype, shape) triples in their order, then every
    expected tensor present."""
    expected = {s.name: s for s in specs}
    seen = set()
    for name, dtype, shape in observed:
        if name in seen:
            raise SchemaError("DuplicateTensor", name)
        seen.add(name)
        spec = expected.get(name)
        if spec is None:
            raise SchemaError("UnexpectedTensor", name)
        if dtype != spec.dtype:
            raise SchemaError("DtypeMismatch", name)
        if tuple(shape) != spec.shape:
            raise SchemaError("ShapeMismatch", name)
    for s in specs:
        if s.name not in seen:
            raise SchemaError("MissingTensor", s.name)


def engine_tensor_names(cfg=None):
    """Checkpoint tensor names in the engine's canonical weight order
    (pvlc_b200.model.init_weights / Weights: vision, projector, decoder)."""
    if cfg is None:
        from .model import ModelConfig
        cfg = ModelConfig()
    e = "visual.vision_model.embeddings"
    vision = [f"{e}.patch_embedding.weight", f"{e}.patch_embedding.bias",
              f"{e}.position_embedding.weight"]
    for layer in range(cfg.vision_layers):
        p = f"visual.vision_model.encoder.layers.{layer}"
        vision += [f"{p}.layer_norm1.weight", f"{p}.layer_norm1.bias"]
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            vision += [f"{p}.self_attn.{proj}.weight", f"{p}.self_attn.{proj}.bias"]
        vision += [f"{p}.layer_norm2.weight", f"{p}.layer_norm2.bias",
                   f"{p}.mlp.fc1.weight", f"{p}.mlp.fc1.bias",
                   f"{p}.mlp.fc2.weight", f"{p}.mlp.fc2.bias"]
    vision += ["visual.vision_model.post_layernorm.weight",
               "visual.vision_model.post_layernorm.bias"]
    projector = ["mlp_AR.pre_norm.weight", "mlp_AR.pre_norm.bias",
                 "mlp_AR.linear_1.weight", "mlp_AR.linear_1.bias",
                 "mlp_AR.linear_2.weight", "mlp_AR.linear_2.bias"]
    decoder = ["model.embed_tokens.weight"]
    for layer in range(cfg.decoder_layers):
        p = f"model.layers.{layer}"
        decoder += [f"{p}.input_layernorm.weight", f"{p}.self_attn.q_proj.weight",
                    f"{p}.self_attn.k_proj.weight", f"{p}.self_attn.v_proj.weight",
                    f"{p}.self_attn.o_proj.weight", f"{p}.post_attention_layernorm.weight",
                    f"{p}.mlp.gate_proj.weight", f"{p}.mlp.up_proj.weight",
                    f"{p}.mlp.down_proj.weight"]
    decoder += ["model.norm.weight", "lm_head.weight"]
    return vision, projector, decoder


# ------------------------------------------------------------------- header writing
def _padded(header: bytes) -> bytes:
    return header + b" " * (-len(header) % 8)


def safetensors_header(entries, metadata=None) -> bytes:
    """A safetensors header as the common writer lays it out: compact JSON,
    ``__metadata__`` first, then each (name, dtype, shape, data_offsets) in the given
    order with fields dtype, shape, data_offsets; padded with spaces to 8 bytes."""
    root = {}
    if metadata is not None:
        root["__metadata__"] = dict(metadata)
    for name, dtype, shape, offsets in entries:
        root[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": list(offsets)}
    return _padded(_compact_json(root))


def name_sorted_layout(specs):
    """(name, dtype, shape, data_offsets) for a payload laid out in name order, as the
    published checkpoint is (lm_head.weight first at offset 0)."""
    entries, off = [], 0
    for s in sorted(specs, key=lambda t: t.name.encode()):
        n = DTYPE_BYTES[s.dtype]
        for d in s.shape:
            n *= d
        entries.append((s.name, s.dtype, s.shape, (off, off + n)))
        off += n
    return entries


def fp16_output_header(catalog: SafetensorsCatalog, source_blake3: str) -> bytes:
    """fp16.rs:403-437: the FP16 checkpoint's header -- the source metadata plus
    pvlc.conversion and pvlc.source_blake3, every tensor as F16 with its source shape and
    offsets; serde_json's sorted-key compact form, padded with spaces to 8 bytes."""
    meta = dict(catalog.metadata)
    meta["pvlc.conversion"] = FP16_CHECKPOINT_CONVERSION_ID
    meta["pvlc.source_blake3"] = source_blake3
    root = {"__metadata__": dict(sorted(meta.items(), key=lambda kv: kv[0].encode()))}
    for t in catalog.tensors:
        root[t.name] = {"data_offsets": list(t.data_offsets), "dtype": "F16",
                        "shape": list(t.shape)}
    root = dict(sorted(root.items(), key=lambda kv: kv[0].encode()))
    return _padded(_compact_json(root))


# ------------------------------------------------------------------- device payload
def _bf16_tensors_in_offset_order(catalog):
    ts = sorted(catalog.tensors, key=lambda t: t.data_offsets)
    for t in ts:
        if t.dtype != "BF16":
            raise Fp16CheckpointError("UnsupportedSourceDtype",
                                      f"source tensor dtype is {t.dtype}, expected BF16", t.name)
    return ts


def _rejection_error(catalog, record: int):
    """Decodes the kernel's rejection word into the reference's error (fp16.rs:230-252)."""
    index, out_of_range = record >> 1, record & 1
    byte = 2 * index
    for t in catalog.tensors:
        if t.data_offsets[0] <= byte < t.data_offsets[1]:
            name, element = t.name, (byte - t.data_offsets[0]) // 2
            break
    else:
        name, element = None, index
    if out_of_range:
        return Fp16CheckpointError("OutOfRangeSource",
                                   "finite BF16 source value is outside finite F16 range",
                                   name, element)
    return Fp16CheckpointError("NonFiniteSource", "BF16 source value is NaN or infinity",
                               name, element)


def _pread_exact(fd, view, offset):
    got = 0
    while got < len(view):
        r = os.preadv(fd, [view[got:]], offset + got)
        if r <= 0:
            raise Fp16CheckpointError("Io", "source checkpoint is truncated")
        got += r


class _DevicePayload:
    """Chunked host -> device pipeline: the payload is read into two pinned buffers in
    turn (each chunk by several threads, one slice each: one thread copying out of the
    page cache reads ~7.5 GB/s), each copied to HBM and converted there in place;
    hashing and the consumer of each converted chunk are optional hooks."""

    READ_SLICE = 8 << 20

    def __init__(self, device, chunk_bytes=DEVICE_CHUNK_BYTES, readers=None):
        import torch
        from . import abi
        abi.lib()
        self.torch, self.abi = torch, abi
        self.device = torch.device(device or "cuda")
        self.chunk = chunk_bytes - chunk_bytes % 16
        self.pinned = [torch.empty(self.chunk, dtype=torch.uint8, pin_memory=True)
                       for _ in range(2)]
        self.ready = [None, None]
        self.word = torch.full((1,), -1, dtype=torch.int64, device=self.device)
        self.readers = readers or max(1, min(8, os.cpu_count() or 1))

    def run(self, fh, body_len, dst=None, on_chunk=None, hasher=None):
        """Reads body_len payload bytes from fh's position (fh's own position is left
        alone).  dst: a device uint8 buffer of body_len bytes to convert into (in place),
        or None to convert through a device chunk buffer handed to
        on_chunk(offset, device_chunk, n)."""
        from concurrent.futures import ThreadPoolExecutor
        torch = self.torch
        stream = torch.cuda.current_stream(self.device)
        scratch = None if dst is not None else torch.empty(self.chunk, dtype=torch.uint8,
                                                           device=self.device)
        fd, base = fh.fileno(), fh.tell()
        # the library launches on the calling thread's current device
        with torch.cuda.device(self.device), ThreadPoolExecutor(self.readers) as pool:
            return self._run(pool, fd, base, body_len, dst, scratch, stream, on_chunk, hasher)

    def _run(self, pool, fd, base, body_len, dst, scratch, stream, on_chunk, hasher):
        torch = self.torch
        for i, off in enumerate(range(0, body_len, self.chunk)):
            slot = i & 1
            if self.ready[slot] is not None:
                self.ready[slot].synchronize()
            n = min(self.chunk, body_len - off)
            host = self.pinned[slot][:n]
            view = memoryview(host.numpy())
            parts = [pool.submit(_pread_exact, fd, view[a:min(n, a + self.READ_SLICE)],
                                 base + off + a) for a in range(0, n, self.READ_SLICE)]
            for f in parts:
                f.result()
            if hasher is not None:
                hasher.update(view)
            target = dst[off:off + n] if dst is not None else scratch[:n]
            target.copy_(host, non_blocking=True)
            self.abi.check(self.abi.lib().pvlc_bf16_to_f16(
                target.data_ptr(), target.data_ptr(), n // 2, off // 2, self.word.data_ptr(),
                stream.cuda_stream), "pvlc_bf16_to_f16")
            if on_chunk is not None:
                on_chunk(off, target, n)
            ev = torch.cuda.Event()
            ev.record(stream)
            self.ready[slot] = ev
        stream.synchronize()
        return int(self.word.item()) & _U64_MAX

    NO_REJECTION = _U64_MAX


def load_payload_f16(catalog: SafetensorsCatalog, device=None, chunk_bytes=DEVICE_CHUNK_BYTES):
    """The whole BF16 payload of a checked catalog converted to fp16 in one device
    buffer (same byte offsets).  Raises Fp16CheckpointError for a non-BF16 tensor (before
    any upload) or for the first rejected element."""
    import torch
    _bf16_tensors_in_offset_order(catalog)
    if catalog.source_path is None:
        raise _fail("SourceUnavailable", "catalog was created from a borrowed reader")
    pipe = _DevicePayload(device, chunk_bytes)
    blob = torch.empty(catalog.body_len + (-catalog.body_len % 16), dtype=torch.uint8,
                       device=pipe.device)
    fh, file_len = _open_regular_file(catalog.source_path)
    with fh:
        if file_len != catalog.file_len:
            raise _fail("DataLengthMismatch", "source file length changed after catalog import")
        fh.seek(catalog.data_start)
        record = pipe.run(fh, catalog.body_len, dst=blob)
    if record != pipe.NO_REJECTION:
        raise _rejection_error(catalog, record)
    return blob


def _tensor_view(blob, t: TensorHeader, shape=None):
    import torch
    start, end = t.data_offsets
    v = blob[start:end]
    if start % 16:
        v = v.clone()
    return v.view(torch.float16).view(*(shape or t.shape))


def load_weights(path, cfg=None, device=None, chunk_bytes=DEVICE_CHUNK_BYTES):
    """A PaddleOCR-VL-1.6 BF16 safetensors checkpoint as the engine's fp16 Weights.
    The header is checked against the exact catalog first (SchemaError); the payload
    is converted on the device (Fp16CheckpointError on a rejected element).  The
    returned tensors are views into one device buffer."""
    from .model import ModelConfig, Weights
    cfg = cfg or ModelConfig()
    catalog = SafetensorsCatalog.open(path)
    catalog.validate_paddleocr_vl_16(cfg)
    blob = load_payload_f16(catalog, device, chunk_bytes)
    vnames, pnames, dnames = engine_tensor_names(cfg)
    patch = catalog.tensor(vnames[0])
    vision = [_tensor_view(blob, patch, (cfg.vision_hidden, cfg.patch_input))]
    vision += [_tensor_view(blob, catalog.tensor(n)) for n in vnames[1:]]
    projector = [_tensor_view(blob, catalog.tensor(n)) for n in pnames]
    decoder = [_tensor_view(blob, catalog.tensor(n)) for n in dnames]
    return Weights(vision, projector, decoder)


def _require_distinct_new_output(source, output):
    """fp16.rs:524-552."""
    src, out = os.path.abspath(source), os.path.abspath(output)
    alias = src == out
    if not alias and os.path.exists(output) and os.path.exists(source):
        alias = os.path.samefile(source, output)
    if alias:
        raise Fp16CheckpointError("SourceDestinationAlias",
                                  "source and output checkpoint paths alias the same file")
    if os.path.lexists(output):
        raise Fp16CheckpointError("OutputAlreadyExists",
                                  f"output checkpoint {output} already exists")


def convert_bf16_checkpoint_to_f16(source, output, device=None,
                                   chunk_bytes=DEVICE_CHUNK_BYTES) -> dict:
    """fp16.rs:278-401 with the payload converted on the GPU: a new FP16 safetensors
    file with the reference's header and payload bits, staged beside the output and
    linked into place only when complete (never overwriting).  Returns the reference's
    conversion report as a dict."""
    import tempfile

    import blake3

    _require_distinct_new_output(source, output)
    try:
        source_len = os.stat(source).st_size
        with open(source, "rb") as fh:
            h = blake3.blake3()
            while chunk := fh.read(16 << 20):
                h.update(chunk)
        source_blake3 = h.hexdigest()
    except OSError as e:
        raise Fp16CheckpointError("Io", f"cannot read source checkpoint {source}: {e}") from e
    try:
        catalog = SafetensorsCatalog.open(source)
    except SafetensorsImportError as e:
        raise Fp16CheckpointError("InvalidSource", str(e), e.tensor_name) from e
    tensors = _bf16_tensors_in_offset_order(catalog)
    header = fp16_output_header(catalog, source_blake3)
    pipe = _DevicePayload(device, chunk_bytes)
    out_hash, src_hash = blake3.blake3(), blake3.blake3()
    parent = os.path.dirname(os.path.abspath(output))
    fd, staged = tempfile.mkstemp(dir=parent, prefix=".pvlc-f16-")
    out_bytes = [0]
    try:
        with os.fdopen(fd, "wb") as out, open(source, "rb") as fh:
            def emit(b):
                out.write(b)
                out_hash.update(b)
                out_bytes[0] += len(b)

            emit(struct.pack("<Q", len(header)))
            emit(header)
            head = fh.read(catalog.data_start)
            src_hash.update(head)
            back = [_empty_pinned(pipe.chunk)]

            def on_chunk(off, dev, n):
                back[0][:n].copy_(dev[:n])          # synchronous D2H of the converted chunk
                emit(memoryview(back[0][:n].numpy()))

            record = pipe.run(fh, catalog.body_len, on_chunk=on_chunk, hasher=src_hash)
            out.flush()
            os.fsync(out.fileno())
        if record != pipe.NO_REJECTION:
            raise _rejection_error(catalog, record)
        if src_hash.hexdigest() != source_blake3 or os.stat(source).st_size != source_len:
            raise Fp16CheckpointError("SourceChanged",
                                      "source checkpoint changed between identity and "
                                      "conversion passes")
        try:
            os.link(staged, output)
        except FileExistsError:
            raise Fp16CheckpointError("OutputAlreadyExists",
                                      f"output checkpoint {output} already exists") from None
    finally:
        if os.path.exists(staged):
            os.unlink(staged)
    return {
        "conversion": FP16_CHECKPOINT_CONVERSION_ID,
        "tensor_count": len(catalog.tensors),
        "element_count": sum(t.byte_len // 2 for t in tensors),
        "source_bytes": source_len,
        "output_bytes": out_bytes[0],
        "source_blake3": source_blake3,
        "output_blake3": out_hash.hexdigest(),
        "max_payload_buffer_bytes": min(pipe.chunk, catalog.body_len),
    }


def _empty_pinned(nbytes):
    import torch
    return torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
