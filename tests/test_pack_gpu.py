"""BLAKE3 on the device (pvlc_blake3) and the .pvlc reader's device-side digest check.

The digests must equal the BLAKE3 reference implementation's bit for bit: the committed
vectors (tests/golden/blake3_vectors.json, input byte i mod 251 across block, chunk and
tree-level boundaries), random data at sizes up to tens of MiB (against the `blake3`
package), unaligned views, and the reference's tiny-pack digest
(crates/pvlc-pack/tests/pack_contract.rs)."""
import json
import os

import blake3
import numpy as np
import pytest
import torch

from pvlc_b200 import ops
from pvlc_b200 import pack as P

from test_pack import TINY_BLAKE3, TINY_LEN, _build, _manifest, _sections

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "blake3_vectors.json")


def _dev_hash(data: bytes, offset: int = 0) -> str:
    """BLAKE3 of `data` placed `offset` bytes into a device buffer."""
    buf = torch.zeros(len(data) + offset + 16, dtype=torch.uint8, device="cuda")
    if data:
        buf[offset:offset + len(data)] = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    return bytes(ops.blake3(buf[offset:offset + len(data)]).cpu().numpy()).hex()


def test_golden_vectors(cuda_lib):
    g = json.load(open(GOLDEN))
    for n, want in g["digests"].items():
        data = bytes(i % 251 for i in range(int(n)))
        assert _dev_hash(data) == want, n
        assert _dev_hash(data, offset=3) == want, f"{n} unaligned"


@pytest.mark.parametrize("n", [1 << 20, (1 << 20) + 17, 3 * (1 << 20) + 1024 * 5 + 9,
                               (37 << 20) + 333])
def test_random_sizes_against_reference_implementation(cuda_lib, n):
    rng = np.random.default_rng(n)
    data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
    assert _dev_hash(data) == blake3.blake3(data).hexdigest()


def test_tiny_pack_digest_and_device_built_pack(cuda_lib):
    host_built = _build()
    assert len(host_built) == TINY_LEN
    assert _dev_hash(host_built) == TINY_BLAKE3
    # the writer's own digests, computed on the device, give the same bytes
    b = P.PackBuilder(_manifest())
    for s in _sections():
        b.add_section(s)
    assert b.build() == host_built


def test_open_verifies_every_section_on_the_device(cuda_lib):
    data = _build()
    r = P.PackReader.open(data)
    for s in _sections():
        t = r.section_tensor(s.id)
        assert t.is_cuda and bytes(t.cpu().numpy()) == s.data
    for e in P.PackReader.parse(data).entries:
        bad = bytearray(data)
        bad[e.offset + e.byte_len // 2] ^= 1
        with pytest.raises(P.PackError) as err:
            P.PackReader.open(bytes(bad))
        assert err.value.code == P.PackErrorCode.ChecksumMismatch, e.id


def test_large_weight_section_round_trip(cuda_lib):
    """A 24 MiB weight shard next to small sections: built and verified on the device."""
    rng = np.random.default_rng(9)
    w = rng.integers(0, 256, 24 << 20, dtype=np.uint8).tobytes()
    b = P.PackBuilder(_manifest())
    b.add_section(P.PackSection("weights.layer_00", P.SectionKind.WeightShard, 4096, w))
    b.add_section(P.PackSection("self_test.probe", P.SectionKind.SelfTest, 16, b"\7" * 33))
    data = b.build()
    assert data == b.build(digest=lambda x: blake3.blake3(x).digest())
    r = P.PackReader.open(data)
    t = r.section_tensor("weights.layer_00")
    assert t.numel() == len(w) and t.data_ptr() % 4096 == r.device_buffer.data_ptr() % 4096
    assert bytes(ops.blake3(t).cpu().numpy()) == blake3.blake3(w).digest()
