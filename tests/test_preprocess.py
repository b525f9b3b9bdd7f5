"""Image preprocessing (pvlc_b200.preprocess) against the reference's vision contract.

Expected values are the literals of crates/pvlc-cpu-ref/tests/vision_contract.rs
(:119-365): the smart-resize boundary table, patch/channel/pixel order, and the
blake3 digests of the bicubic outputs that the reference pinned to the official
Python image processor.
"""
import blake3
import numpy as np
import pytest

from pvlc_b200 import preprocess as P

PATCH = 14


def test_smart_resize_matches_pinned_processor_at_geometry_boundaries():
    # vision_contract.rs:128-153
    for h, w, expected in [(1, 1, (336, 336)), (27, 27, (336, 336)), (28, 28, (336, 336)),
                           (29, 29, (336, 336)), (300, 800, (308, 812)), (800, 300, (812, 308)),
                           (350, 350, (336, 336)), (3000, 3000, (980, 980))]:
        assert P.smart_resize(h, w) == expected, (h, w)
    h, w = P.smart_resize(300, 800)
    assert (h // PATCH) * (w // PATCH) == 1276


def test_smart_resize_of_config_image_is_980():
    # 1024 x 1024 -> 980 x 980 -> 70 x 70 patches -> 1225 merged tokens
    assert P.smart_resize(1024, 1024) == (980, 980)


def test_smart_resize_rejects_invalid_geometry_and_config():
    # vision_contract.rs:155-188
    for h, w in [(0, 28), (28, 0), (28, 28 * 201)]:
        with pytest.raises(P.PreprocessError) as e:
            P.smart_resize(h, w)
        assert e.value.code == P.INVALID_IMAGE_GEOMETRY
    for bad in [P.VisionPreprocessConfig(patch_size=0), P.VisionPreprocessConfig(merge_size=0),
                P.VisionPreprocessConfig(min_pixels=1000, max_pixels=999)]:
        with pytest.raises(P.PreprocessError) as e:
            P.smart_resize(28, 28, bad)
        assert e.value.code == P.INVALID_PREPROCESS_CONFIG


def test_patch_channel_and_pixel_order():
    # vision_contract.rs:190-235
    h, w = 28, 56
    y, x, c = np.meshgrid(np.arange(h), np.arange(w), np.arange(3), indexing="ij")
    rgb = ((y * 31 + x * 17 + c * 53) % 256).astype(np.uint8)
    cfg = P.VisionPreprocessConfig(min_pixels=h * w, max_pixels=h * w)
    out = P.canonical_rgb8_to_patches(rgb, cfg)
    assert (out.resized_height, out.resized_width) == (h, w)
    assert out.image_grid_thw == (1, 2, 4)
    vals = out.values.reshape(-1)
    assert vals.size == 8 * 3 * PATCH * PATCH
    for py in range(2):
        for px in range(4):
            patch = py * 4 + px
            for ch in range(3):
                src = rgb[py * PATCH:(py + 1) * PATCH, px * PATCH:(px + 1) * PATCH, ch]
                exp = (np.float32(2.0) * src.astype(np.float32) / np.float32(255.0)
                       - np.float32(1.0))
                got = vals[(patch * 3 + ch) * PATCH * PATCH:(patch * 3 + ch + 1) * PATCH * PATCH]
                assert np.array_equal(got, exp.reshape(-1))


def _formula_image(h, w):
    y, x = np.meshgrid(np.arange(h), np.arange(w), indexing="ij")
    rgb = np.empty((h, w, 3), np.uint8)
    rgb[..., 0] = (x * 17 + y * 3) % 256
    rgb[..., 1] = (x * 5 + y * 29 + 7) % 256
    rgb[..., 2] = (x * 11 + y * 13 + 19) % 256
    return rgb


def test_bicubic_downscale_matches_official_processor_digest():
    # vision_contract.rs:237-283
    rgb = _formula_image(29, 31)
    cfg = P.VisionPreprocessConfig(min_pixels=28 * 28, max_pixels=28 * 28)
    out = P.canonical_rgb8_to_patches(rgb, cfg)
    assert (out.resized_height, out.resized_width) == (28, 28)
    assert out.image_grid_thw == (1, 2, 2)
    vals = out.values.reshape(-1)
    assert blake3.blake3(vals.astype("<f4").tobytes()).hexdigest() == \
        "d7319132258c207228f7d1c6544e6b5d08bf285ab4deaabdd32335c4ca541994"
    bits = vals.view(np.uint32)
    for i, b in [(0, 0xbf7dfdfe), (13, 0x3f79f9fa), (196, 0xbf6feff0), (588, 0xbd888888),
                 (1500, 0x3f0b8b8c), (2351, 0x3f119192)]:
        assert int(bits[i]) == b, i


def test_bicubic_production_upscale_matches_official_processor_digest():
    # vision_contract.rs:285-340
    rgb = _formula_image(29, 31)
    assert blake3.blake3(rgb.tobytes()).hexdigest() == \
        "cb6acd67be313b63eaf51641695a424a52a0dc63287dc195792ce447a179837d"
    out = P.canonical_rgb8_to_patches(rgb)
    assert (out.resized_height, out.resized_width) == (336, 364)
    assert out.image_grid_thw == (1, 24, 26)
    vals = out.values.reshape(-1)
    assert vals.size == 366_912
    assert blake3.blake3(vals.astype("<f4").tobytes()).hexdigest() == \
        "54cc35abbf418aee73fb775ce963f3f3edee9da33fbcba137b583735706a8a4e"
    bits = vals.view(np.uint32)
    for i, b in [(0, 0xbf800000), (13, 0xbf6bebec), (588, 0xbf67e7e8), (10_000, 0xbea2a2a2),
                 (100_000, 0xbf0b8b8c), (300_000, 0x3de8e8f0), (366_911, 0x3f19999a)]:
        assert int(bits[i]) == b, i


def test_constant_image_stays_constant_across_mandatory_upscale():
    # vision_contract.rs:342-353
    out = P.canonical_rgb8_to_patches(np.array([[[0, 128, 255]]], np.uint8))
    assert (out.resized_height, out.resized_width) == (336, 336)
    assert out.image_grid_thw == (1, 24, 24)
    v = out.values.reshape(-1, 3, PATCH * PATCH)
    exp = [np.float32(-1.0), np.float32(2.0) * np.float32(128.0) / np.float32(255.0) -
           np.float32(1.0), np.float32(1.0)]
    for ch in range(3):
        assert np.all(v[:, ch] == exp[ch])


def test_wrong_buffer_shape_is_rejected():
    with pytest.raises(P.PreprocessError) as e:
        P.canonical_rgb8_to_patches(np.zeros((2, 2, 2), np.uint8))
    assert e.value.code == P.DIMENSION_MISMATCH
