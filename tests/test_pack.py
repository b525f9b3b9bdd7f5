"""The .pvlc pack writer and reader, host side (no GPU): byte-exact against the reference's
tiny-pack fixture and every rejection rule of PackReader::open except the section digests
(crates/pvlc-pack/tests/pack_contract.rs).  The digests here come from the `blake3`
package as the checker; tests/test_pack_gpu.py checks the device digests."""
import struct

import blake3
import pytest

from pvlc_b200 import pack as P

# crates/pvlc-pack/tests/pack_contract.rs: the tiny pack's length and BLAKE3
TINY_LEN = 841
TINY_BLAKE3 = "01fe6f47b810877d4c2bb17bc68d4c4aef1fee4d21fc7216837d4005251346c6"


def _digest(b):
    return blake3.blake3(b).digest()


def _manifest():
    return P.PackManifest(P.MODEL_ID, P.MODEL_REVISION, P.COMPILER_MODEL_ABI, "a" * 64,
                          "fidelity", [[28, 28], [56, 84]], 128)


def _sections():
    return [
        P.PackSection("weights.tiny", P.SectionKind.WeightShard, 256,
                      bytes((i * 17 + 3) % 256 for i in range(73))),
        P.PackSection("self_test.tiny", P.SectionKind.SelfTest, 16,
                      bytes([0xff, 0x00, 0x7f, 0x80, 0x01])),
        P.PackSection("ir.semantic", P.SectionKind.SemanticIr, 64, b'{"nodes":[]}\n'),
    ]


def _build(order=(0, 1, 2)):
    b = P.PackBuilder(_manifest())
    secs = _sections()
    for i in order:
        b.add_section(secs[i])
    return b.build(digest=_digest)


def _code(data):
    with pytest.raises(P.PackError) as e:
        P.PackReader.parse(data)
    return e.value.code


def _entries(data):
    """(entry start, id start, id end, padding end, offset, byte_len) of each entry."""
    mlen, = struct.unpack_from("<I", data, 12)
    count, = struct.unpack_from("<I", data, 20)
    cur, out = P.HEADER_BYTES + mlen, []
    for _ in range(count):
        idl, = struct.unpack_from("<H", data, cur)
        off, blen = struct.unpack_from("<QQ", data, cur + 8)
        ids = cur + P.DIRECTORY_FIXED_BYTES
        end = cur + (P.DIRECTORY_FIXED_BYTES + idl + 7) // 8 * 8
        out.append((cur, ids, ids + idl, end, off, blen))
        cur = end
    return out


def test_tiny_pack_is_byte_exact_and_order_independent():
    first = _build((0, 1, 2))
    assert first == _build((2, 0, 1))
    assert len(first) == TINY_LEN
    assert blake3.blake3(first).hexdigest() == TINY_BLAKE3


def test_parse_round_trip():
    r = P.PackReader.parse(_build((1, 2, 0)))
    assert r.manifest == _manifest()
    assert [e.id for e in r.entries] == ["ir.semantic", "self_test.tiny", "weights.tiny"]
    assert bytes(r.section("ir.semantic")) == b'{"nodes":[]}\n'
    assert bytes(r.section("self_test.tiny")) == bytes([0xff, 0x00, 0x7f, 0x80, 0x01])
    assert bytes(r.section("weights.tiny")) == _sections()[0].data
    assert r.entries[0].kind == P.SectionKind.SemanticIr
    assert r.entries[2].alignment == 256 and len(r.entries[2].digest) == 32
    assert r.entries[2].digest == _digest(_sections()[0].data)
    assert r.section("missing") is None


def test_manifest_identity_and_compiler_build():
    m = P.PackManifest.paddleocr_vl_16("a" * 64)
    assert (m.model_id, m.model_revision, m.compiler_model_abi, m.precision_profile) == \
        (P.MODEL_ID, P.MODEL_REVISION, P.COMPILER_MODEL_ABI, "fidelity")
    for bad in ("a" * 63, "a" * 65, "A" * 64, "g" * 64):
        with pytest.raises(P.PackError) as e:
            P.PackManifest.paddleocr_vl_16(bad)
        assert e.value.code == P.PackErrorCode.InvalidCompilerBuild


def test_builder_rejections():
    for field, value in (("model_id", "other/model"), ("model_revision", "0" * 40),
                         ("compiler_model_abi", P.COMPILER_MODEL_ABI + 1)):
        m = _manifest()
        setattr(m, field, value)
        with pytest.raises(P.PackError) as e:
            P.PackBuilder(m).build(digest=_digest)
        assert e.value.code == P.PackErrorCode.ModelIdentityMismatch
    b = P.PackBuilder(_manifest())
    b.add_section(_sections()[0])
    with pytest.raises(P.PackError) as e:
        b.add_section(_sections()[0])
    assert e.value.code == P.PackErrorCode.DuplicateSection
    for a in (0, 3, 8192):
        with pytest.raises(P.PackError) as e:
            P.PackBuilder(_manifest()).add_section(
                P.PackSection("weights.bad", P.SectionKind.WeightShard, a, b"\1"))
        assert e.value.code == P.PackErrorCode.InvalidAlignment
    for a in (1, 4096):
        b = P.PackBuilder(_manifest())
        b.add_section(P.PackSection(f"weights.valid_{a}", P.SectionKind.WeightShard, a, b"\1"))
        P.PackReader.parse(b.build(digest=_digest))
    with pytest.raises(P.PackError) as e:
        P.PackBuilder(_manifest()).add_section(
            P.PackSection("Bad.Id", P.SectionKind.SelfTest, 8, b"\1"))
    assert e.value.code == P.PackErrorCode.InvalidSectionId


def test_reader_rejects_header_length_and_padding_faults():
    pristine = _build()
    bad = bytearray(pristine)
    bad[0] ^= 1
    assert _code(bytes(bad)) == P.PackErrorCode.BadMagic
    bad = bytearray(pristine)
    bad[8:12] = struct.pack("<I", 2)
    assert _code(bytes(bad)) == P.PackErrorCode.UnsupportedVersion
    for n in range(P.HEADER_BYTES):
        assert _code(pristine[:n]) == P.PackErrorCode.Truncated
    assert _code(pristine[:-1]) == P.PackErrorCode.LengthMismatch
    assert _code(pristine + b"\0") == P.PackErrorCode.LengthMismatch
    bad = bytearray(pristine)
    bad[24:32] = struct.pack("<Q", len(pristine) - 1)
    assert _code(bytes(bad)) == P.PackErrorCode.LengthMismatch
    ents = _entries(pristine)
    for _, _, id_end, pad_end, _, _ in ents:
        assert id_end < pad_end
        bad = bytearray(pristine)
        bad[id_end] = 1
        assert _code(bytes(bad)) == P.PackErrorCode.NonZeroPadding
    mlen, dlen = struct.unpack_from("<II", pristine, 12)
    prev_end = P.HEADER_BYTES + mlen + dlen
    for _, _, _, _, off, blen in ents:
        assert prev_end < off
        bad = bytearray(pristine)
        bad[prev_end] = 1
        assert _code(bytes(bad)) == P.PackErrorCode.NonZeroPadding
        prev_end = off + blen


def test_reader_rejects_malformed_directory():
    pristine = _build()
    mlen, = struct.unpack_from("<I", pristine, 12)
    first = P.HEADER_BYTES + mlen
    bad = bytearray(pristine)
    bad[first + 3] = 1
    assert _code(bytes(bad)) == P.PackErrorCode.InvalidDirectory
    bad = bytearray(pristine)
    bad[first + 4:first + 8] = struct.pack("<I", 3)
    assert _code(bytes(bad)) == P.PackErrorCode.InvalidAlignment
    bad = bytearray(pristine)
    off, = struct.unpack_from("<Q", pristine, first + 8)
    bad[first + 8:first + 16] = struct.pack("<Q", off + 1)
    assert _code(bytes(bad)) == P.PackErrorCode.InvalidSectionLayout
    bad = bytearray(pristine)
    bad[first + 2] = 255
    assert _code(bytes(bad)) == P.PackErrorCode.UnknownSectionKind
    bad = bytearray(pristine)
    bad[_entries(pristine)[0][1]] = 0xff
    assert _code(bytes(bad)) == P.PackErrorCode.InvalidDirectory
    for count in (2, 4):
        bad = bytearray(pristine)
        bad[20:24] = struct.pack("<I", count)
        assert _code(bytes(bad)) == P.PackErrorCode.InvalidDirectory
    bad = bytearray(pristine)
    _, ids, ide, _, _, _ = _entries(pristine)[0]
    assert ide - ids == len(b"zz.semantic")
    bad[ids:ide] = b"zz.semantic"
    assert _code(bytes(bad)) == P.PackErrorCode.NonCanonicalDirectory


def test_reader_survives_hostile_lengths_counts_offsets_and_overlaps():
    pristine = _build()
    for lo in (12, 16, 20):
        bad = bytearray(pristine)
        bad[lo:lo + 4] = struct.pack("<I", 0xFFFFFFFF)
        assert _code(bytes(bad)) == P.PackErrorCode.InvalidHeader
    bad = bytearray(pristine)
    bad[24:32] = struct.pack("<Q", 2**64 - 1)
    assert _code(bytes(bad)) == P.PackErrorCode.LengthMismatch
    ents = _entries(pristine)
    first, second = ents[0][0], ents[1][0]
    bad = bytearray(pristine)
    bad[first:first + 2] = struct.pack("<H", 0xFFFF)
    assert _code(bytes(bad)) == P.PackErrorCode.InvalidDirectory
    for lo in (first + 8, first + 16):
        bad = bytearray(pristine)
        bad[lo:lo + 8] = struct.pack("<Q", 2**64 - 1)
        assert _code(bytes(bad)) == P.PackErrorCode.InvalidSectionLayout
    bad = bytearray(pristine)
    bad[second + 8:second + 16] = struct.pack("<Q", ents[0][4])
    assert _code(bytes(bad)) == P.PackErrorCode.InvalidSectionLayout
    bad = bytearray(pristine)
    bad[second + 16:second + 24] = struct.pack("<Q", 2**64 - 1)
    assert _code(bytes(bad)) == P.PackErrorCode.InvalidSectionLayout


def test_reader_rejects_duplicate_ids_and_noncanonical_manifest():
    b = P.PackBuilder(_manifest())
    b.add_section(P.PackSection("test.aaaa", P.SectionKind.SelfTest, 8, b"\1"))
    b.add_section(P.PackSection("test.bbbb", P.SectionKind.SelfTest, 8, b"\2"))
    data = bytearray(b.build(digest=_digest))
    (_, i0, e0, _, _, _), (_, i1, e1, _, _, _) = _entries(bytes(data))
    data[i1:e1] = data[i0:e0]
    assert _code(bytes(data)) == P.PackErrorCode.DuplicateSection
    # a manifest with a space added (same length budget: rebuild the header around it)
    pristine = _build()
    mlen, dlen = struct.unpack_from("<II", pristine, 12)
    raw = pristine[P.HEADER_BYTES:P.HEADER_BYTES + mlen]
    spaced = raw.replace(b'":', b'": ', 1)
    assert spaced != raw
    body = pristine[P.HEADER_BYTES + mlen:]
    hdr = bytearray(pristine[:P.HEADER_BYTES])
    hdr[12:16] = struct.pack("<I", len(spaced))
    hdr[24:32] = struct.pack("<Q", len(pristine) + 1)
    assert _code(bytes(hdr) + spaced + body) == P.PackErrorCode.InvalidManifest
