"""Checkpoint import, host side: the safetensors catalog, the exact model schema and the
BF16 -> F16 rule, against the reference's own contract tests (restated; paths relative
to the reference project root).  No GPU: the device conversion is in
tests/test_checkpoint_gpu.py."""
import io
import json
import os
import struct

import blake3
import numpy as np
import pytest

import pvlc_oracle as O
from pvlc_b200 import abi
from pvlc_b200 import checkpoint as C
from pvlc_b200.model import ModelConfig


def container(header_json: bytes, body: bytes) -> bytes:
    # crates/pvlc-safetensors/tests/importer_contract.rs:16-37
    header = header_json + b" " * (-len(header_json) % 8)
    return struct.pack("<Q", len(header)) + header + body


def write(tmp_path, header_json: bytes, body: bytes, name="fixture.safetensors"):
    p = tmp_path / name
    p.write_bytes(container(header_json, body))
    return p


def code_of(fn):
    with pytest.raises((C.SafetensorsImportError, C.SchemaError, C.Fp16CheckpointError)) as e:
        fn()
    return e.value.code


# ------------------------------------------------------------------ schema (exact catalog)
def test_schema_is_the_reference_catalog_byte_for_byte():
    # crates/pvlc-model-schema/tests/schema_contract.rs:8-13,417-493
    specs = C.schema_specs()
    assert len(specs) == 620
    names = [s.name for s in specs]
    assert names == sorted(names) and len(set(names)) == 620
    assert len({s.semantic_id for s in specs}) == 620
    assert all(s.dtype == "BF16" for s in specs)
    cat = C.canonical_catalog_bytes(specs)
    assert len(cat) == 58_966 and cat.endswith(b"\n")
    assert blake3.blake3(cat).hexdigest() == \
        "422b0532712a71baee6d085de1fc79f057764f2fee71545c18a680d1b97543a6"
    sem = C.canonical_semantic_map_bytes(specs)
    assert len(sem) == 68_676
    assert blake3.blake3(sem).hexdigest() == \
        "749a6e5c7d91013b13b4e77cb967a078015ba9b3f791e582f04c791beff086b7"
    assert C.MODEL_ID == "PaddlePaddle/PaddleOCR-VL-1.6"
    assert C.MODEL_REVISION == "66317acc4c9fc17bd154591ce650735cd2855f3e"


def test_schema_validator_reports_each_mutation():
    # schema_contract.rs:576-640
    specs = C.schema_specs()
    exact = [(s.name, s.dtype, s.shape) for s in specs]
    C.validate_schema(exact, specs)
    cases = [
        (exact + [("unexpected.weight", "BF16", (1,))], "UnexpectedTensor", "unexpected.weight"),
        (exact + [exact[3]], "DuplicateTensor", exact[3][0]),
        ([(n, "F16" if i == 7 else d, s) for i, (n, d, s) in enumerate(exact)], "DtypeMismatch",
         exact[7][0]),
        ([(n, d, tuple(reversed(s)) if i == 0 else s) for i, (n, d, s) in enumerate(exact)],
         "ShapeMismatch", exact[0][0]),
        (exact[:100] + exact[101:], "MissingTensor", exact[100][0]),
    ]
    for observed, code, name in cases:
        with pytest.raises(C.SchemaError) as e:
            C.validate_schema(observed, specs)
        assert (e.value.code, e.value.tensor_name) == (code, name)


def test_published_checkpoint_layout_and_sparse_open(tmp_path):
    """importer_contract.rs:130-168 records the published file's layout: 1,917,255,968
    bytes, a 78,488-byte header, lm_head.weight at [0, 211812352] and
    visual.vision_model.post_layernorm.weight last at [1917175168, 1917177472].  The
    name-ordered writer reproduces all of it, and opening a sparse file of that size
    reads the header only (:338-354)."""
    entries = C.name_sorted_layout(C.schema_specs())
    header = C.safetensors_header(entries, {"format": "pt"})
    assert len(header) == 78_488
    body = entries[-1][3][1]
    assert 8 + len(header) + body == 1_917_255_968
    p = tmp_path / "model.safetensors"
    with open(p, "wb") as f:
        f.write(struct.pack("<Q", len(header)) + header)
        f.truncate(8 + len(header) + body)
    cat = C.SafetensorsCatalog.open(p)
    assert (cat.file_len, cat.header_len, len(cat.tensors)) == (1_917_255_968, 78_488, 620)
    assert cat.metadata == {"format": "pt"}
    cat.validate_paddleocr_vl_16()
    assert cat.tensor("lm_head.weight").data_offsets == (0, 211_812_352)
    assert cat.tensor("visual.vision_model.post_layernorm.weight").data_offsets == \
        (1_917_175_168, 1_917_177_472)


def test_engine_weight_order_covers_the_checkpoint():
    """The engine's canonical weight lists name checkpoint tensors one to one; the 12
    tensors it does not read are the packing position table and the pooling head."""
    for cfg in (ModelConfig(), ModelConfig(vision_layers=2, decoder_layers=3, vocab=512)):
        v, p, d = C.engine_tensor_names(cfg)
        assert len(v) == 3 + 16 * cfg.vision_layers + 2
        assert len(p) == 6 and len(d) == 1 + 9 * cfg.decoder_layers + 2
        spec = {s.name for s in C.schema_specs(cfg)}
        used = v + p + d
        assert len(set(used)) == len(used) and set(used) <= spec
        unused = sorted(spec - set(used))
        assert len(unused) == 12
        assert all(n.startswith("visual.vision_model.head.") or "packing_position" in n
                   for n in unused)


# ------------------------------------------------------------------ importer contract
def test_imports_sorted_catalog_and_streams_exact_bytes(tmp_path):
    # importer_contract.rs:46-82
    p = write(tmp_path, b'{"__metadata__":{"format":"pt","producer":"contract-test"},'
              b'"z":{"dtype":"F32","shape":[1],"data_offsets":[4,8]},'
              b'"a":{"dtype":"BF16","shape":[2],"data_offsets":[0,4]}}', bytes(range(8)))
    cat = C.SafetensorsCatalog.open(p)
    assert cat.file_len == os.path.getsize(p) and cat.header_len % 8 == 0
    assert [t.name for t in cat.tensors] == ["a", "z"]
    a = cat.tensors[0]
    assert (a.dtype, a.shape, a.data_offsets, a.byte_len) == ("BF16", (2,), (0, 4), 4)
    assert cat.metadata["format"] == "pt"
    buf = io.BytesIO()
    assert cat.copy_tensor_to("z", buf) == 4 and buf.getvalue() == bytes([4, 5, 6, 7])
    with pytest.raises(C.SafetensorsImportError) as e:
        cat.copy_tensor_to("missing", io.BytesIO())
    assert (e.value.code, e.value.tensor_name) == ("TensorNotFound", "missing")
    with open(p, "rb") as fh:
        borrowed = C.SafetensorsCatalog.read_from(fh, os.path.getsize(p))
    assert code_of(lambda: borrowed.copy_tensor_to("a", io.BytesIO())) == "SourceUnavailable"


def test_materializes_bf16_f16_f32_bits_exactly(tmp_path):
    # importer_contract.rs:83-127 (+ an F16 tensor: lib.rs:420-438 keeps NaN payloads)
    body = b"".join(struct.pack("<H", b) for b in (0x0000, 0x3F80, 0xBF20, 0x7F7F))
    body += b"".join(struct.pack("<f", v) for v in (0.5, -2.25, np.pi, -0.0))
    body += bytes([7])
    body += b"".join(struct.pack("<H", b) for b in (0x0001, 0x7C01, 0xFC00, 0x3C00, 0x8400))
    p = write(tmp_path, b'{"bf":{"dtype":"BF16","shape":[4],"data_offsets":[0,8]},'
              b'"fp":{"dtype":"F32","shape":[2,2],"data_offsets":[8,24]},'
              b'"byte":{"dtype":"U8","shape":[1],"data_offsets":[24,25]},'
              b'"h":{"dtype":"F16","shape":[5],"data_offsets":[25,35]}}', body)
    cat = C.SafetensorsCatalog.open(p)
    assert cat.load_tensor_f32("bf").view(np.uint32).tolist() == \
        [0x00000000, 0x3F800000, 0xBF200000, 0x7F7F0000]
    assert cat.load_tensor_f32("fp").view(np.uint32).tolist() == \
        np.array([0.5, -2.25, np.pi, -0.0], np.float32).view(np.uint32).tolist()
    assert cat.load_tensor_f32("h").view(np.uint32).tolist() == \
        [0x33800000, 0x7F802000, 0xFF800000, 0x3F800000, 0xB8800000]
    assert code_of(lambda: cat.load_tensor_f32("byte")) == "UnsupportedTensorConversion"
    assert code_of(lambda: cat.load_tensor_f32("missing")) == "TensorNotFound"


def test_schema_mismatch_comes_from_the_model_check(tmp_path):
    # importer_contract.rs:170-182
    p = write(tmp_path, b'{"lm_head.weight":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]}}',
              b"\0\0")
    with pytest.raises(C.SchemaError) as e:
        C.SafetensorsCatalog.open(p).validate_paddleocr_vl_16()
    assert (e.value.code, e.value.tensor_name) == ("ShapeMismatch", "lm_head.weight")


def test_rejects_truncated_oversized_unaligned_headers(tmp_path):
    # importer_contract.rs:184-228
    assert C.MAX_HEADER_BYTES == 100_000_000
    cases = [(bytes(range(1, 8)), "HeaderPrefixTruncated"),
             (struct.pack("<Q", C.MAX_HEADER_BYTES + 8), "HeaderTooLarge"),
             (struct.pack("<Q", (1 << 64) - 1), "HeaderTooLarge"),
             (struct.pack("<Q", 7) + b"{}     ", "HeaderLengthNotAligned"),
             (struct.pack("<Q", 16) + b"{}      ", "HeaderTruncated")]
    for i, (raw, code) in enumerate(cases):
        p = tmp_path / f"c{i}.safetensors"
        p.write_bytes(raw)
        assert code_of(lambda: C.SafetensorsCatalog.open(p)) == code


@pytest.mark.parametrize("header,body,code", [
    # importer_contract.rs:229-261
    (b'{\xff}', b"", "InvalidHeaderUtf8"),
    (b'{"a":}', b"", "InvalidHeaderJson"),
    (b'{"a":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]},'
     b'"a":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]}}', b"\0\0", "DuplicateHeaderKey"),
    (b'{"a":{"dtype":"BF16","dtype":"F16","shape":[1],"data_offsets":[0,2]}}', b"\0\0",
     "DuplicateHeaderKey"),
    # :262-288
    (b'{"a":{"dtype":"BF16","shape":[1],"data_offsets":[0,2],"surprise":true}}', b"\0\0",
     "InvalidTensorMetadata"),
    (b'{"__metadata__":{"format":7}}', b"", "InvalidMetadata"),
    (b'{"a":{"dtype":"F128","shape":[1],"data_offsets":[0,16]}}', bytes(16), "UnsupportedDtype"),
    # :289-336
    (b'{"a":{"dtype":"BF16","shape":[18446744073709551615,2],"data_offsets":[0,0]}}', b"",
     "ShapeElementCountOverflow"),
    (b'{"a":{"dtype":"BF16","shape":[2],"data_offsets":[0,2]}}', b"\0\0",
     "TensorByteLengthMismatch"),
    (b'{"a":{"dtype":"U8","shape":[2],"data_offsets":[0,2]},'
     b'"b":{"dtype":"U8","shape":[2],"data_offsets":[1,3]}}', bytes(3), "OverlappingData"),
    (b'{"a":{"dtype":"U8","shape":[1],"data_offsets":[0,1]},'
     b'"b":{"dtype":"U8","shape":[1],"data_offsets":[2,3]}}', bytes(3), "NonContiguousData"),
    (b'{"a":{"dtype":"U8","shape":[1],"data_offsets":[0,1]}}', bytes(2), "DataLengthMismatch"),
    # field-type rules of the tensor visitor (lib.rs:708-803)
    (b'{"a":{"shape":[1],"data_offsets":[0,2]}}', b"\0\0", "InvalidTensorMetadata"),
    (b'{"a":{"dtype":"BF16","shape":[-1],"data_offsets":[0,2]}}', b"\0\0",
     "InvalidTensorMetadata"),
    (b'{"a":{"dtype":"BF16","shape":[1.0],"data_offsets":[0,2]}}', b"\0\0",
     "InvalidTensorMetadata"),
    (b'{"a":{"dtype":"BF16","shape":[true],"data_offsets":[0,2]}}', b"\0\0",
     "InvalidTensorMetadata"),
    (b'{"a":{"dtype":"BF16","shape":[1],"data_offsets":[0,2,4]}}', b"\0\0",
     "InvalidTensorMetadata"),
    (b'{"a":{"dtype":"BF16","shape":[1],"data_offsets":[2,0]}}', b"\0\0", "InvalidDataOffsets"),
    (b'{"":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]}}', b"\0\0", "InvalidTensorMetadata"),
    (b'{"a":{"dtype":"BF16","shape":[NaN],"data_offsets":[0,2]}}', b"\0\0", "InvalidHeaderJson"),
    (b'[1,2]', b"", "InvalidHeaderJson"),
])
def test_rejects_malformed_headers(tmp_path, header, body, code):
    p = write(tmp_path, header, body)
    assert code_of(lambda: C.SafetensorsCatalog.open(p)) == code


def test_rejects_symlinks_and_non_regular_files(tmp_path):
    # importer_contract.rs:439-461
    real = write(tmp_path, b"{}", b"")
    link = tmp_path / "link.safetensors"
    os.symlink(real, link)
    assert code_of(lambda: C.SafetensorsCatalog.open(link)) == "NotRegularFile"
    assert code_of(lambda: C.SafetensorsCatalog.open(tmp_path)) == "NotRegularFile"
    assert code_of(lambda: C.SafetensorsCatalog.open(tmp_path / "absent")) == "Io"
    assert C.SafetensorsCatalog.open(real).tensors == []


# ------------------------------------------------------------------ BF16 -> F16 rule
def test_bf16_to_f16_known_answers_and_rejections():
    # crates/pvlc-safetensors/tests/fp16_checkpoint_conversion_contract.rs:57-87
    kat = [(0x0000, 0x0000), (0x8000, 0x8000), (0x3F80, 0x3C00), (0xBF80, 0xBC00),
           (0x3880, 0x0400), (0x3800, 0x0200), (0x3380, 0x0001), (0x3300, 0x0000),
           (0x33C0, 0x0002), (0xB3C0, 0x8002), (0x477F, 0x7BF8)]
    out, status = O.bf16_to_f16_bits([a for a, _ in kat])
    assert status.tolist() == [0] * len(kat)
    assert out.tolist() == [b for _, b in kat]
    _, status = O.bf16_to_f16_bits([0x4780, 0xC780, 0x7F80, 0xFF80, 0x7FC1, 0xFFC1])
    assert status.tolist() == [2, 2, 1, 1, 1, 1]


def test_bf16_to_f16_rule_is_ieee_rne_on_every_pattern():
    """All 65,536 BF16 patterns: the restated rule equals IEEE round-to-nearest-even
    (numpy's f32 -> f16) wherever it converts, and rejects exactly exponent 0xff and
    magnitudes of 2^16 and above."""
    bits = np.arange(1 << 16, dtype=np.uint16)
    out, status = O.bf16_to_f16_bits(bits)
    values = (bits.astype(np.uint32) << 16).view(np.float32)
    ok = status == 0
    assert np.array_equal(values[ok].astype(np.float16).view(np.uint16), out[ok])
    assert np.array_equal(status == 1, ~np.isfinite(values))
    assert np.array_equal(status == 2, np.isfinite(values) & (np.abs(values) >= 65536.0))


def test_stream_form_stops_at_the_first_rejection():
    # fp16.rs:212-276: the element index names the first rejected element in order
    src = np.full(40, 0x3F80, np.uint16)
    src[[17, 23]] = [0x4780, 0x7F80]
    out, err = O.stream_bf16_to_f16(src)
    assert out is None and err == (17, 2)
    out, err = O.stream_bf16_to_f16(np.full(9, 0xBF80, np.uint16))
    assert err is None and out.tolist() == [0xBC00] * 9


# ------------------------------------------------------------------ FP16 output header
def test_fp16_output_header_matches_the_reference_fixture():
    """fp16_checkpoint_conversion_contract.rs:44-56,89-180: the converted file keeps
    every tensor's shape and offsets as F16 and adds pvlc.conversion and
    pvlc.source_blake3 to the source metadata; keys are written sorted."""
    src = container(b'{"__metadata__":{"format":"pt","owner":"contract"},'
                    b'"z":{"dtype":"BF16","shape":[4],"data_offsets":[0,8]},'
                    b'"a":{"dtype":"BF16","shape":[5],"data_offsets":[8,18]}}', bytes(18))
    cat = C.SafetensorsCatalog.read_from(io.BytesIO(src), len(src))
    digest = blake3.blake3(src).hexdigest()
    header = C.fp16_output_header(cat, digest)
    assert len(header) % 8 == 0
    text = header.decode().rstrip(" ")
    assert text.startswith('{"__metadata__":{"format":"pt","owner":"contract",'
                           '"pvlc.conversion":"bf16_to_ieee_f16_rne_v1","pvlc.source_blake3":"')
    assert text.endswith('"a":{"data_offsets":[8,18],"dtype":"F16","shape":[5]},'
                         '"z":{"data_offsets":[0,8],"dtype":"F16","shape":[4]}}')
    out = struct.pack("<Q", len(header)) + header + bytes(18)
    back = C.SafetensorsCatalog.read_from(io.BytesIO(out), len(out))
    assert [(t.name, t.dtype, t.shape, t.data_offsets) for t in back.tensors] == \
        [("a", "F16", (5,), (8, 18)), ("z", "F16", (4,), (0, 8))]
    assert back.metadata["pvlc.source_blake3"] == digest
    assert json.loads(text)["__metadata__"]["owner"] == "contract"


def test_library_exports_the_conversion_entry_point():
    assert "pvlc_bf16_to_f16" in abi.EXPORTED
    assert hasattr(abi.lib(), "pvlc_bf16_to_f16")


def test_payload_reader_fills_slices_exactly(tmp_path):
    """The device pipeline's reader threads each fill one slice of a pinned chunk with
    positional reads; a short file is an Io error, never a partial chunk."""
    data = bytes(range(256)) * 1000
    p = tmp_path / "payload.bin"
    p.write_bytes(data)
    buf = bytearray(1000)
    with open(p, "rb") as f:
        C._pread_exact(f.fileno(), memoryview(buf), 12_345)
        assert bytes(buf) == data[12_345:13_345]
        with pytest.raises(C.Fp16CheckpointError) as e:
            C._pread_exact(f.fileno(), memoryview(buf), len(data) - 10)
    assert e.value.code == "Io"


def test_converter_refuses_before_touching_a_device(tmp_path):
    """fp16.rs:278-305,524-552: aliasing, an existing output, an unreadable catalog and a
    non-BF16 tensor are refused on the host, before any payload work, leaving no file."""
    src = write(tmp_path, b'{"w":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]}}', b"\x80\x3f",
                "source.safetensors")
    existing = tmp_path / "existing.safetensors"
    existing.write_bytes(b"keep")
    cases = [(src, src, "SourceDestinationAlias"),
             (src, existing, "OutputAlreadyExists"),
             (write(tmp_path, b'{"w":{"dtype":"BF16","shape":[2],"data_offsets":[0,2]}}',
                    b"\0\0", "bad.safetensors"), tmp_path / "bad.out", "InvalidSource"),
             (write(tmp_path, b'{"w":{"dtype":"F16","shape":[1],"data_offsets":[0,2]}}',
                    b"\0\x3c", "f16.safetensors"), tmp_path / "f16.out",
              "UnsupportedSourceDtype")]
    for source, output, code in cases:
        with pytest.raises(C.Fp16CheckpointError) as e:
            C.convert_bf16_checkpoint_to_f16(source, output)
        assert e.value.code == code
    assert existing.read_bytes() == b"keep"
    assert not (tmp_path / "bad.out").exists() and not (tmp_path / "f16.out").exists()
    assert not [p for p in os.listdir(tmp_path) if p.startswith(".pvlc-f16-")]
