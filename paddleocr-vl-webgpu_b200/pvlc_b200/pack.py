"""Checksummed .pvlc model packs: reader and writer of the reference's format, with the
section digests computed on the B200.

Format (crates/pvlc-pack/src/lib.rs:1-713, `PackBuilder::build` / `PackReader::open`):

    header (32 B)   magic "PVLCPK01" | version u32 = 1 | manifest_len u32 | directory_len u32
                    | section_count u32 | file_len u64                      (little endian)
    manifest        canonical JSON (keys in byte order, no spaces) + "\\n"
    directory       per section, sorted by id: id_len u16 | kind tag u8 | 0 u8 | alignment u32
                    | offset u64 | byte_len u64 | blake3(section) 32 B | id, zero-padded to 8 B
    sections        each at the next multiple of its alignment, zero padding between them

The reader runs the reference's checks in the reference's order and raises `PackError`
with the same code names (`PackErrorCode`); the last check, every section's BLAKE3 digest,
runs on the device: the pack is copied to HBM once and `pvlc_blake3` hashes each section in
place, so the weights are verified where they are used.  The writer builds byte-identical
packs (the reference's tiny pack, 841 bytes, is a test fixture).
"""
from __future__ import annotations

import dataclasses
import enum
import json
import struct

PACK_MAGIC = b"PVLCPK01"
PACK_FORMAT_VERSION = 1
HEADER_BYTES = 32
DIRECTORY_FIXED_BYTES = 56
MAX_MANIFEST_BYTES = 1_048_576
MAX_DIRECTORY_BYTES = 16_777_216
MAX_SECTIONS = 65_536
MAX_ALIGNMENT = 4_096
MAX_SECTION_ID_BYTES = 128

# the pinned model identity (crates/pvlc-model-schema/src/lib.rs:12-14)
MODEL_ID = "PaddlePaddle/PaddleOCR-VL-1.6"
MODEL_REVISION = "66317acc4c9fc17bd154591ce650735cd2855f3e"
COMPILER_MODEL_ABI = 1


class PackErrorCode(enum.Enum):
    """crates/pvlc-pack/src/lib.rs PackErrorCode, in declaration order."""
    ModelIdentityMismatch = 0
    InvalidCompilerBuild = 1
    InvalidManifest = 2
    InvalidSectionId = 3
    DuplicateSection = 4
    InvalidAlignment = 5
    BadMagic = 6
    UnsupportedVersion = 7
    Truncated = 8
    LengthMismatch = 9
    InvalidHeader = 10
    InvalidDirectory = 11
    UnknownSectionKind = 12
    NonCanonicalDirectory = 13
    InvalidSectionLayout = 14
    ChecksumMismatch = 15
    NonZeroPadding = 16


class PackError(Exception):
    def __init__(self, code: PackErrorCode, message: str):
        super().__init__(f"pack error {code.name}: {message}")
        self.code = code
        self.message = message


class SectionKind(enum.IntEnum):
    """Directory tags (crates/pvlc-pack/src/lib.rs SectionKind::tag)."""
    SemanticIr = 1
    WeightShard = 2
    SelfTest = 3
    ModelSchema = 4
    SemanticMap = 5


PRECISION_PROFILES = ("fidelity", "balanced", "turbo")


def _align_up(value: int, alignment: int) -> int:
    return (value + alignment - 1) // alignment * alignment


def _check_alignment(alignment: int):
    if not (0 < alignment <= MAX_ALIGNMENT and alignment & (alignment - 1) == 0):
        raise PackError(PackErrorCode.InvalidAlignment, f"invalid section alignment {alignment}")


def _is_lower_hex_64(value) -> bool:
    return isinstance(value, str) and len(value) == 64 and all(c in "0123456789abcdef" for c in value)


def _semantic_segment(seg: str) -> bool:
    # crates/pvlc-ir/src/lib.rs valid_segment: two digits, or [a-z][a-z0-9_]*
    if seg.isascii() and seg.isdigit():
        return len(seg) == 2
    return (bool(seg) and "a" <= seg[0] <= "z" and
            all("a" <= c <= "z" or "0" <= c <= "9" or c == "_" for c in seg[1:]))


def _artifact_segment(seg: str) -> bool:
    return (bool(seg) and "a" <= seg[0] <= "z" and
            all("a" <= c <= "z" or "0" <= c <= "9" or c in "_-" for c in seg[1:]))


def valid_section_id(sid: str) -> bool:
    """A SemanticId (pvlc-ir) or an artifact id: dot-separated lowercase segments."""
    if not sid or len(sid.encode()) > MAX_SECTION_ID_BYTES:
        return False
    segs = sid.split(".")
    return all(_semantic_segment(s) for s in segs) or all(_artifact_segment(s) for s in segs)


@dataclasses.dataclass
class PackManifest:
    model_id: str
    model_revision: str
    compiler_model_abi: int
    compiler_build: str
    precision_profile: str
    resolution_buckets: list
    context_limit: int

    @classmethod
    def paddleocr_vl_16(cls, compiler_build: str) -> "PackManifest":
        m = cls(MODEL_ID, MODEL_REVISION, COMPILER_MODEL_ABI, compiler_build, "fidelity",
                [[28, 28]], 4096)
        m.validate()
        return m

    def validate(self):
        if (self.model_id != MODEL_ID or self.model_revision != MODEL_REVISION or
                self.compiler_model_abi != COMPILER_MODEL_ABI):
            raise PackError(PackErrorCode.ModelIdentityMismatch,
                            "pack manifest does not identify the pinned PaddleOCR-VL model")
        if not _is_lower_hex_64(self.compiler_build):
            raise PackError(PackErrorCode.InvalidCompilerBuild,
                            "compiler build must be exactly 64 lowercase hexadecimal characters")
        if (self.context_limit == 0 or not self.resolution_buckets or
                any(b[0] == 0 or b[1] == 0 for b in self.resolution_buckets)):
            raise PackError(PackErrorCode.InvalidManifest,
                            "context limit and resolution buckets must be nonzero")

    def canonical_bytes(self) -> bytes:
        """The manifest's one byte form: keys in byte order, compact, then a newline."""
        self.validate()
        doc = {
            "compiler_build": self.compiler_build,
            "compiler_model_abi": self.compiler_model_abi,
            "context_limit": self.context_limit,
            "model_id": self.model_id,
            "model_revision": self.model_revision,
            "precision_profile": self.precision_profile,
            "resolution_buckets": [[int(a), int(b)] for a, b in self.resolution_buckets],
        }
        return json.dumps(doc, separators=(",", ":"), ensure_ascii=False).encode() + b"\n"


def _u32(v) -> bool:
    return type(v) is int and 0 <= v <= 0xFFFFFFFF


def _parse_manifest(raw: bytes) -> PackManifest:
    bad = lambda msg: PackError(PackErrorCode.InvalidManifest, msg)  # noqa: E731
    if not raw.endswith(b"\n"):
        raise bad("canonical manifest must end in one newline")
    try:
        text = raw.decode("utf-8")
    except UnicodeDecodeError:
        raise bad("manifest is not UTF-8") from None
    try:
        doc = json.loads(text)
    except ValueError as e:
        raise bad(f"invalid manifest JSON: {e}") from None
    keys = {"compiler_build", "compiler_model_abi", "context_limit", "model_id",
            "model_revision", "precision_profile", "resolution_buckets"}
    if not isinstance(doc, dict) or set(doc) != keys:
        raise bad("invalid manifest JSON: missing or unknown fields")
    buckets = doc["resolution_buckets"]
    if (not isinstance(doc["compiler_build"], str) or not isinstance(doc["model_id"], str) or
            not isinstance(doc["model_revision"], str) or
            not _u32(doc["compiler_model_abi"]) or not _u32(doc["context_limit"]) or
            doc["precision_profile"] not in PRECISION_PROFILES or not isinstance(buckets, list) or
            not all(isinstance(b, list) and len(b) == 2 and all(_u32(x) for x in b)
                    for b in buckets)):
        raise bad("invalid manifest JSON: field types")
    m = PackManifest(doc["model_id"], doc["model_revision"], doc["compiler_model_abi"],
                     doc["compiler_build"], doc["precision_profile"], buckets,
                     doc["context_limit"])
    if m.canonical_bytes() != raw:
        raise bad("manifest JSON is not in canonical byte form")
    return m


@dataclasses.dataclass
class PackSection:
    id: str
    kind: SectionKind
    alignment: int
    data: bytes


@dataclasses.dataclass
class PackEntry:
    id: str
    kind: SectionKind
    alignment: int
    offset: int
    byte_len: int
    digest: bytes


def device_digests(buf, spans):
    """BLAKE3 of each (offset, length) span of a CUDA uint8 tensor, computed on the device;
    returns the 32-byte digests (one device-to-host copy)."""
    import torch
    from . import ops
    if not spans:
        return []
    out = torch.empty((len(spans), 32), dtype=torch.uint8, device=buf.device)
    need = max(int(ops.abi.lib().pvlc_blake3_workspace_bytes(n)) for _, n in spans)
    ws = torch.empty(need, dtype=torch.uint8, device=buf.device)
    for i, (off, n) in enumerate(spans):
        ops.blake3(buf[off:off + n], digest=out[i], workspace=ws)
    host = out.cpu().numpy()
    return [bytes(host[i]) for i in range(len(spans))]


def _upload(data, device):
    import torch
    host = torch.frombuffer(bytearray(data), dtype=torch.uint8) if len(data) else \
        torch.empty(0, dtype=torch.uint8)
    return host.pin_memory().to(device, non_blocking=False)


class PackBuilder:
    """crates/pvlc-pack/src/lib.rs PackBuilder: sections keyed by id, emitted in id order."""

    def __init__(self, manifest: PackManifest):
        self.manifest = manifest
        self.sections: dict = {}

    def add_section(self, section: PackSection):
        if not valid_section_id(section.id):
            raise PackError(PackErrorCode.InvalidSectionId, f"invalid section ID {section.id!r}")
        _check_alignment(section.alignment)
        if section.id in self.sections:
            raise PackError(PackErrorCode.DuplicateSection, f"section {section.id!r} is duplicated")
        self.sections[section.id] = section

    def build(self, digest=None, device="cuda") -> bytes:
        """The pack's bytes.  digest: bytes -> 32-byte BLAKE3 for each section; by default
        every section is hashed on `device` by pvlc_blake3."""
        mbytes = self.manifest.canonical_bytes()
        secs = [self.sections[k] for k in sorted(self.sections)]
        dir_len = sum(_align_up(DIRECTORY_FIXED_BYTES + len(s.id.encode()), 8) for s in secs)
        cursor = HEADER_BYTES + len(mbytes) + dir_len
        offsets = []
        for s in secs:
            cursor = _align_up(cursor, s.alignment)
            offsets.append(cursor)
            cursor += len(s.data)
        if digest is None:
            body = b"".join(bytes(s.data) for s in secs)
            starts, acc = [], 0
            for s in secs:
                starts.append(acc)
                acc += len(s.data)
            digests = device_digests(_upload(body, device),
                                     [(a, len(s.data)) for a, s in zip(starts, secs)])
        else:
            digests = [bytes(digest(bytes(s.data))) for s in secs]
        directory = bytearray()
        for s, off, dg in zip(secs, offsets, digests):
            sid = s.id.encode()
            directory += struct.pack("<HBBIQQ", len(sid), int(s.kind), 0, s.alignment, off,
                                     len(s.data))
            directory += dg + sid
            directory += b"\0" * (_align_up(len(directory), 8) - len(directory))
        out = bytearray(PACK_MAGIC)
        out += struct.pack("<IIIIQ", PACK_FORMAT_VERSION, len(mbytes), dir_len, len(secs), cursor)
        out += mbytes + directory
        for s, off in zip(secs, offsets):
            out += b"\0" * (off - len(out))
            out += bytes(s.data)
        return bytes(out)


class PackReader:
    """crates/pvlc-pack/src/lib.rs PackReader::open, with the digests checked on the device.

    `PackReader.parse(data)` runs every check except the digests (host only);
    `PackReader.open(data, device)` also copies the pack to `device` and compares each
    section's BLAKE3, computed there, with its directory entry; the device copy stays
    available (`section_tensor`)."""

    def __init__(self, data, manifest, entries, device_buffer=None):
        self._data = memoryview(data)
        self.manifest = manifest
        self.entries = entries
        self._by_id = {e.id: e for e in entries}
        self.device_buffer = device_buffer

    @classmethod
    def parse(cls, data) -> "PackReader":
        b = bytes(data)
        n = len(b)
        if n < HEADER_BYTES:
            raise PackError(PackErrorCode.Truncated, "pack is shorter than its fixed header")
        if b[:8] != PACK_MAGIC:
            raise PackError(PackErrorCode.BadMagic, "pack magic mismatch")
        version, mlen, dlen, count, flen = struct.unpack_from("<IIIIQ", b, 8)
        if version != PACK_FORMAT_VERSION:
            raise PackError(PackErrorCode.UnsupportedVersion, f"unsupported pack version {version}")
        if flen != n:
            raise PackError(PackErrorCode.LengthMismatch,
                            f"header declares {flen} bytes but input has {n}")
        if mlen > MAX_MANIFEST_BYTES or dlen > MAX_DIRECTORY_BYTES or count > MAX_SECTIONS:
            raise PackError(PackErrorCode.InvalidHeader,
                            "manifest, directory, or section count exceeds its bound")
        mend = HEADER_BYTES + mlen
        dend = mend + dlen
        if dend > n:
            raise PackError(PackErrorCode.InvalidHeader,
                            "manifest and directory extend beyond the pack")
        manifest = _parse_manifest(b[HEADER_BYTES:mend])

        bad_dir = lambda msg: PackError(PackErrorCode.InvalidDirectory, msg)  # noqa: E731
        entries, cursor, prev = [], mend, None
        for _ in range(count):
            fixed_end = cursor + DIRECTORY_FIXED_BYTES
            if fixed_end > dend:
                raise bad_dir("directory entry fixed fields are truncated")
            id_len, tag, reserved, align, off, blen = struct.unpack_from("<HBBIQQ", b, cursor)
            digest = b[cursor + 24:cursor + 56]
            if reserved != 0:
                raise bad_dir("directory reserved byte is nonzero")
            try:
                kind = SectionKind(tag)
            except ValueError:
                raise PackError(PackErrorCode.UnknownSectionKind,
                                f"unknown section kind tag {tag}") from None
            _check_alignment(align)
            if id_len == 0 or id_len > MAX_SECTION_ID_BYTES:
                raise bad_dir("section ID length is out of bounds")
            id_end = fixed_end + id_len
            entry_end = cursor + _align_up(DIRECTORY_FIXED_BYTES + id_len, 8)
            if entry_end > dend:
                raise bad_dir("section ID or entry padding is truncated")
            try:
                sid = b[fixed_end:id_end].decode("utf-8")
            except UnicodeDecodeError:
                raise bad_dir("section ID is not valid UTF-8") from None
            if not valid_section_id(sid):
                raise bad_dir(f"invalid section ID {sid!r}")
            if any(b[id_end:entry_end]):
                raise PackError(PackErrorCode.NonZeroPadding,
                                "canonical pack padding contains a nonzero byte")
            if prev is not None:
                if sid.encode() == prev.encode():
                    raise PackError(PackErrorCode.DuplicateSection,
                                    f"directory repeats section {sid!r}")
                if sid.encode() < prev.encode():
                    raise PackError(PackErrorCode.NonCanonicalDirectory,
                                    "section IDs are not in canonical byte order")
            prev = sid
            entries.append(PackEntry(sid, kind, align, off, blen, digest))
            cursor = entry_end
        if cursor != dend:
            raise bad_dir("section count does not consume the complete directory")

        layout = lambda: PackError(  # noqa: E731
            PackErrorCode.InvalidSectionLayout,
            "section offsets are noncanonical, overlapping, or out of bounds")
        prev_end = dend
        for e in entries:
            if e.offset != _align_up(prev_end, e.alignment) or e.offset + e.byte_len > n:
                raise layout()
            if any(b[prev_end:e.offset]):
                raise PackError(PackErrorCode.NonZeroPadding,
                                "canonical pack padding contains a nonzero byte")
            prev_end = e.offset + e.byte_len
        if prev_end != n:
            raise layout()
        return cls(b, manifest, entries)

    @classmethod
    def open(cls, data, device="cuda") -> "PackReader":
        r = cls.parse(data)
        buf = _upload(r._data, device)
        got = device_digests(buf, [(e.offset, e.byte_len) for e in r.entries])
        for e, dg in zip(r.entries, got):
            if dg != e.digest:
                raise PackError(PackErrorCode.ChecksumMismatch,
                                f"section {e.id!r} checksum mismatch")
        r.device_buffer = buf
        return r

    def section(self, sid: str):
        """The section's bytes (a view of the pack), or None."""
        e = self._by_id.get(sid)
        return None if e is None else self._data[e.offset:e.offset + e.byte_len]

    def section_tensor(self, sid: str):
        """The section as a CUDA uint8 tensor view of the verified device copy, or None."""
        e = self._by_id.get(sid)
        if e is None or self.device_buffer is None:
            return None
        return self.device_buffer[e.offset:e.offset + e.byte_len]
