"""Checkpoint import on the GPU: the pvlc_bf16_to_f16 kernel (through the C ABI) against
the CPU restatement of the reference's rule, and the loader / converter built on it.

Integer work, so the bar is bit-exact: every converted element equals the oracle's (and
torch's IEEE round-to-nearest-even conversion), and the rejection word names the
element the reference's stream converter stops at
(crates/pvlc-safetensors/src/fp16.rs:171-276)."""
import io
import os
import struct

import numpy as np
import pytest
import torch

import pvlc_oracle as O
from pvlc_b200 import abi
from pvlc_b200 import checkpoint as C
from pvlc_b200 import model as M

pytestmark = pytest.mark.gpu
NONE = (1 << 64) - 1


def convert(src_bits, dst=None, index_base=0, word=None, count=None):
    """One pvlc_bf16_to_f16 call on device int16 tensors; returns (dst, word, status)."""
    if dst is None:
        dst = torch.empty_like(src_bits)
    if word is None:
        word = torch.full((1,), -1, dtype=torch.int64, device=src_bits.device)
    st = abi.lib().pvlc_bf16_to_f16(src_bits.data_ptr(), dst.data_ptr(),
                                    src_bits.numel() if count is None else count, index_base,
                                    word.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return dst, word, st


def record(word):
    torch.cuda.synchronize()
    return int(word.item()) & NONE


def test_every_bf16_pattern_matches_the_oracle(cuda_lib):
    bits = np.arange(1 << 16, dtype=np.uint16)
    ref, status = O.bf16_to_f16_bits(bits)
    ok = status == 0
    dev = torch.from_numpy(bits[ok].view(np.int16)).cuda()
    out, word, st = convert(dev)
    assert st == abi.OK and record(word) == NONE
    assert np.array_equal(out.cpu().numpy().view(np.uint16), ref[ok])
    # all patterns: the word names the first rejected one (0x4780 = 2^16, out of range)
    _, word, st = convert(torch.from_numpy(bits.view(np.int16)).cuda())
    first = int(np.flatnonzero(~ok)[0])
    assert st == abi.OK and first == 0x4780 and record(word) == (first << 1 | 1)


def test_payload_in_place_in_chunks_with_a_ragged_tail(cuda_lib):
    n = 3_000_003
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    vals = torch.randn(n, generator=g, device="cuda") * torch.exp2(
        torch.randint(-30, 14, (n,), generator=g, device="cuda").float())
    src = vals.to(torch.bfloat16).view(torch.int16)
    ref = src.view(torch.bfloat16).to(torch.float16).view(torch.int16)
    host = src.cpu().numpy().view(np.uint16)
    oref, ostat = O.bf16_to_f16_bits(host)
    assert (ostat == 0).all()
    assert np.array_equal(ref.cpu().numpy().view(np.uint16), oref)
    buf = src.clone()
    word = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    cut = 1_234_568                      # chunk edge at a multiple of 8 elements
    for base, count in ((0, cut), (cut, n - cut)):
        piece = buf[base:base + count]
        _, _, st = convert(piece, piece, base, word)
        assert st == abi.OK
    assert record(word) == NONE
    assert torch.equal(buf, ref)
    # plant a NaN and an overflow in the second chunk: the word names the NaN's index
    bad = src.clone()
    bad[2_700_001] = 0x7FC1
    bad[2_900_000] = 0x4780
    word.fill_(-1)
    for base, count in ((0, cut), (cut, n - cut)):
        convert(bad[base:base + count], None, base, word)
    assert record(word) == (2_700_001 << 1)
    _, err = O.stream_bf16_to_f16(bad.cpu().numpy().view(np.uint16))
    assert err == (2_700_001, 1)


@pytest.mark.parametrize("n", [1, 7, 8, 9, 4095, 4096 * 1184 + 5])
def test_odd_lengths(cuda_lib, n):
    rng = np.random.default_rng(n)
    bits = rng.integers(0, 1 << 16, n, dtype=np.uint16)
    bits = np.where(((bits >> 7) & 0xFF) >= 0x8F, bits & 0x83FF, bits).astype(np.uint16)
    ref, status = O.bf16_to_f16_bits(bits)
    assert (status == 0).all()
    out, word, st = convert(torch.from_numpy(bits.view(np.int16)).cuda())
    assert st == abi.OK and record(word) == NONE
    assert np.array_equal(out.cpu().numpy().view(np.uint16), ref)


def test_host_rejects_bad_arguments_without_a_launch(cuda_lib):
    src = torch.zeros(64, dtype=torch.int16, device="cuda")
    word = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    lib, s = abi.lib(), torch.cuda.current_stream().cuda_stream
    assert lib.pvlc_bf16_to_f16(src.data_ptr(), src.data_ptr(), 0, 0, word.data_ptr(), s) == \
        abi.ZERO_DIMENSION
    assert lib.pvlc_bf16_to_f16(None, src.data_ptr(), 8, 0, word.data_ptr(), s) == \
        abi.NULL_POINTER
    assert lib.pvlc_bf16_to_f16(src.data_ptr(), src.data_ptr(), 8, 0, None, s) == \
        abi.NULL_POINTER
    assert lib.pvlc_bf16_to_f16(src.data_ptr() + 2, src.data_ptr(), 8, 0, word.data_ptr(),
                                s) == abi.MISALIGNED_POINTER
    assert lib.pvlc_bf16_to_f16(src.data_ptr(), src.data_ptr(), 8, 1 << 63, word.data_ptr(),
                                s) == abi.ARITHMETIC_OVERFLOW
    assert record(word) == NONE


# ---------------------------------------------------------------- loader and converter
# fewer layers and narrower MLPs than the published model; the vocabulary stays whole
# because the OCR prompt's special tokens have ids above 100,000
SMALL = M.ModelConfig(vision_layers=2, decoder_layers=2, intermediate=512,
                      vision_intermediate=512)


def _write_checkpoint(path, cfg, seed=0, poison=None):
    """A BF16 checkpoint of cfg's exact catalog, payload in name order; norm scales near
    1, everything else N(0, 0.02^2).  Returns {name: device bf16 tensor}."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    entries = C.name_sorted_layout(C.schema_specs(cfg))
    tensors = {}
    with open(path, "wb") as f:
        header = C.safetensors_header(entries, {"format": "pt"})
        f.write(struct.pack("<Q", len(header)) + header)
        for name, _, shape, _ in entries:
            x = torch.randn(shape, generator=g, device="cuda")
            x = 1 + 0.1 * x if ("norm" in name and name.endswith("weight")) else 0.02 * x
            t = x.to(torch.bfloat16)
            if poison and name == poison[0]:
                t.view(-1).view(torch.int16)[poison[1]] = poison[2]
            tensors[name] = t
            f.write(t.view(torch.int16).cpu().numpy().tobytes())
    return tensors


def test_load_weights_is_bit_exact_and_drives_the_engine(cuda_lib, tmp_path):
    path = tmp_path / "small.safetensors"
    src = _write_checkpoint(path, SMALL)
    w = C.load_weights(path, SMALL, chunk_bytes=8 << 20)
    names = C.engine_tensor_names(SMALL)
    loaded = w.vision + w.projector + w.decoder
    ref_lists = []
    for part in names:
        ref_lists.append([src[n].to(torch.float16) for n in part])
    ref_lists[0][0] = ref_lists[0][0].reshape(SMALL.vision_hidden, SMALL.patch_input)
    for name, got, ref in zip(sum(names, []), loaded, sum(ref_lists, [])):
        assert got.dtype == torch.float16 and got.shape == ref.shape, name
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), name
        assert got.data_ptr() % 16 == 0, name
    rng = np.random.default_rng(1)
    page = rng.integers(0, 256, (112, 140, 3), dtype=np.uint8)
    from pvlc_b200 import preprocess as P
    pcfg = P.VisionPreprocessConfig(min_pixels=112 * 140, max_pixels=112 * 140)
    a = M.OcrEngine.from_checkpoint(path, SMALL).recognize([page], max_new_tokens=6,
                                                          preprocess_config=pcfg)
    b = M.OcrEngine(SMALL, M.Weights(*ref_lists)).recognize([page], max_new_tokens=6,
                                                           preprocess_config=pcfg)
    ta = [[int(x) for x in t] for t in a["tokens"]]
    tb = [[int(x) for x in t] for t in b["tokens"]]
    assert ta == tb and len(ta[0]) >= 1


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible GPUs")
def test_load_onto_a_device_that_is_not_current(cuda_lib, tmp_path):
    """cuda:0 stays current while the weights go to cuda:1: the conversion kernels
    must run on cuda:1 (the loader makes it current around its launches), the
    result must live there and be bit-exact."""
    path = tmp_path / "small.safetensors"
    src = _write_checkpoint(path, SMALL, seed=3)
    torch.cuda.set_device(0)
    w = C.load_weights(path, SMALL, device="cuda:1", chunk_bytes=8 << 20)
    assert torch.cuda.current_device() == 0
    names = sum(C.engine_tensor_names(SMALL), [])
    for name, got in zip(names, w.vision + w.projector + w.decoder):
        assert got.device == torch.device("cuda:1"), name
        ref = src[name].to(torch.float16).reshape(got.shape).to("cuda:1")
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), name
    blob = C.load_payload_f16(C.SafetensorsCatalog.open(path), "cuda:1")
    assert blob.device == torch.device("cuda:1")


def test_load_weights_names_the_first_rejected_element(cuda_lib, tmp_path):
    path = tmp_path / "poisoned.safetensors"
    _write_checkpoint(path, SMALL, seed=2,
                      poison=("model.layers.1.mlp.down_proj.weight", 12345, 0x7F80))
    with pytest.raises(C.Fp16CheckpointError) as e:
        C.load_weights(path, SMALL, chunk_bytes=4 << 20)
    assert (e.value.code, e.value.tensor_name, e.value.element_index) == \
        ("NonFiniteSource", "model.layers.1.mlp.down_proj.weight", 12345)
    with pytest.raises(C.SchemaError) as e:
        C.load_weights(path, M.ModelConfig())       # wrong catalog: checked before any upload
    assert e.value.code in ("ShapeMismatch", "MissingTensor")


def _container(path, header_json: bytes, body: bytes):
    header = header_json + b" " * (-len(header_json) % 8)
    path.write_bytes(struct.pack("<Q", len(header)) + header + body)


def _bf16(values):
    return b"".join(struct.pack("<H", v) for v in values)


def test_convert_checkpoint_file_matches_the_reference_contract(cuda_lib, tmp_path):
    # crates/pvlc-safetensors/tests/fp16_checkpoint_conversion_contract.rs:44-56,89-180
    source = tmp_path / "source.safetensors"
    _container(source, b'{"__metadata__":{"format":"pt","owner":"contract"},'
               b'"z":{"dtype":"BF16","shape":[4],"data_offsets":[0,8]},'
               b'"a":{"dtype":"BF16","shape":[5],"data_offsets":[8,18]}}',
               _bf16([0x0000, 0x8000, 0x3F80, 0xBF80]) +
               _bf16([0x3880, 0x3800, 0x3380, 0x33C0, 0x477F]))
    before = source.read_bytes()
    first, second = tmp_path / "first.safetensors", tmp_path / "second.safetensors"
    r1 = C.convert_bf16_checkpoint_to_f16(source, first)
    r2 = C.convert_bf16_checkpoint_to_f16(source, second)
    assert source.read_bytes() == before
    assert first.read_bytes() == second.read_bytes() and r1 == r2
    import blake3
    assert r1["conversion"] == C.FP16_CHECKPOINT_CONVERSION_ID
    assert (r1["tensor_count"], r1["element_count"]) == (2, 9)
    assert r1["source_bytes"] == len(before)
    assert r1["source_blake3"] == blake3.blake3(before).hexdigest()
    assert r1["output_blake3"] == blake3.blake3(first.read_bytes()).hexdigest()
    assert r1["output_bytes"] == len(first.read_bytes())
    out = C.SafetensorsCatalog.open(first)
    assert all(t.dtype == "F16" for t in out.tensors)
    assert out.tensor("z").data_offsets == (0, 8) and out.tensor("a").data_offsets == (8, 18)
    assert out.metadata["owner"] == "contract" and out.metadata["format"] == "pt"
    assert out.metadata["pvlc.source_blake3"] == r1["source_blake3"]
    raw = io.BytesIO()
    out.copy_tensor_to("a", raw)
    assert raw.getvalue() == _bf16([0x0400, 0x0200, 0x0001, 0x0002, 0x7BF8])
    assert out.load_tensor_f32("z").view(np.uint32).tolist() == \
        [0x00000000, 0x80000000, 0x3F800000, 0xBF800000]
    # refuses aliasing and existing outputs (:381-391)
    with pytest.raises(C.Fp16CheckpointError) as e:
        C.convert_bf16_checkpoint_to_f16(source, source)
    assert e.value.code == "SourceDestinationAlias"
    with pytest.raises(C.Fp16CheckpointError) as e:
        C.convert_bf16_checkpoint_to_f16(source, first)
    assert e.value.code == "OutputAlreadyExists"


def test_convert_rejections_leave_no_output(cuda_lib, tmp_path):
    # fp16_checkpoint_conversion_contract.rs:291-380
    cases = [("wrong-dtype", "F16", 0x3C00, "UnsupportedSourceDtype"),
             ("positive-infinity", "BF16", 0x7F80, "NonFiniteSource"),
             ("negative-infinity", "BF16", 0xFF80, "NonFiniteSource"),
             ("nan", "BF16", 0x7FC1, "NonFiniteSource"),
             ("overflow", "BF16", 0x4780, "OutOfRangeSource")]
    for name, dtype, bits, code in cases:
        source, output = tmp_path / f"{name}.safetensors", tmp_path / f"{name}.fp16.safetensors"
        _container(source, ('{"weight":{"dtype":"%s","shape":[1],"data_offsets":[0,2]}}'
                            % dtype).encode(), _bf16([bits]))
        with pytest.raises(C.Fp16CheckpointError) as e:
            C.convert_bf16_checkpoint_to_f16(source, output)
        assert (e.value.code, e.value.tensor_name) == (code, "weight")
        if code != "UnsupportedSourceDtype":
            assert e.value.element_index == 0
        assert not output.exists()
    late = tmp_path / "late"
    late.mkdir()
    count = C.COPY_BUFFER_BYTES // 2 + 1
    source, output = late / "late-failure.safetensors", late / "late-failure.fp16.safetensors"
    body = bytearray(2 * count)
    body[-2:] = _bf16([0x7F80])
    _container(source, ('{"weight":{"dtype":"BF16","shape":[%d],"data_offsets":[0,%d]}}'
                        % (count, 2 * count)).encode(), bytes(body))
    with pytest.raises(C.Fp16CheckpointError) as e:
        C.convert_bf16_checkpoint_to_f16(source, output, chunk_bytes=4096)
    assert (e.value.code, e.value.tensor_name, e.value.element_index) == \
        ("NonFiniteSource", "weight", count - 1)
    assert sorted(os.listdir(late)) == ["late-failure.safetensors"]
