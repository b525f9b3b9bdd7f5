"""Multi-process request sharding on CPU ranks (gloo, world_size 2).

The "device" work of each rank is the CPU oracle's decode step, so the test
exercises the sharding, the gather and the failure handling without a GPU.
A rank that raises before the gather must make the other rank's collective
end with an error within the process-group timeout, not hang.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _request(i):
    """Deterministic decode request i -> output digest (oracle on CPU)."""
    import pvlc_oracle as O
    from pvlc_b200 import positions
    rng = np.random.default_rng(100 + i)
    L = 20 + 7 * i
    cap = L + 4
    cos, sin = positions.linear_rope_tables(cap)
    q = rng.standard_normal(16 * 128).astype(np.float32)
    kn = rng.standard_normal(2 * 128).astype(np.float32)
    vn = rng.standard_normal(2 * 128).astype(np.float32)
    kc = rng.standard_normal((cap, 2, 128)).astype(np.float32)
    vc = rng.standard_normal((cap, 2, 128)).astype(np.float32)
    out = O.decode_step(q, kn, vn, cos, sin, L, kc, vc, L)
    return float(np.abs(out).sum())


def _worker(rank, world, port, mode, result_q):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "paddleocr-vl-webgpu_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    from pvlc_b200 import dist as pd
    import torch.distributed as tdist
    pd.init("gloo", timeout_s=10.0)
    try:
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure on rank 1")
        if mode == "tokens":
            # 5 requests over 2 ranks (shards of 3 and 2); request i emits i + 1 ids
            mine = pd.shard(5, rank, world)
            toks = [[100 * i + j for j in range(i + 1)] for i in mine]
            merged = pd.gather_token_ids(toks, 5, 8)
            result_q.put((rank, "ok", merged, None))
            return
        merged = pd.run_sharded(6, _request, rank, world)
        t = pd.max_over_ranks(float(rank + 1))
        result_q.put((rank, "ok", merged, t))
    except Exception as e:   # noqa: BLE001 - reported to the parent
        result_q.put((rank, "error", type(e).__name__ + ": " + str(e)[:200], None))
    finally:
        try:
            tdist.destroy_process_group()
        except Exception:
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2):
        rank, status, payload, t = q.get(timeout=120)
        results[rank] = (status, payload, t)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_two_rank_sharding_matches_single_process():
    sys.path.insert(0, os.path.join(ROOT, "paddleocr-vl-webgpu_b200"))
    from pvlc_b200 import dist as pd
    assert pd.shard(6, 0, 2) == [0, 2, 4] and pd.shard(6, 1, 2) == [1, 3, 5]
    assert pd.shard(5, 1, 3) == [1, 4]
    with pytest.raises(ValueError):
        pd.shard(4, 2, 2)
    res = _run("ok")
    status, merged, t = res[0]
    assert status == "ok", merged
    assert res[1][0] == "ok" and res[1][1] is None    # only rank 0 receives the gather
    assert t == 2.0 and res[1][2] == 2.0              # max over ranks
    expected = {i: _request(i) for i in range(6)}
    assert merged == expected


def test_failed_rank_ends_the_peer_collective_with_an_error():
    res = _run("fail")
    assert res[1][0] == "error" and "injected failure" in res[1][1]
    # rank 0 must not hang: its gather fails once rank 1 is gone
    assert res[0][0] == "error"


def test_token_ids_gather_to_rank0_by_request_index():
    sys.path.insert(0, os.path.join(ROOT, "paddleocr-vl-webgpu_b200"))
    from pvlc_b200 import dist as pd
    res = _run("tokens")
    assert res[0][0] == "ok" and res[1][0] == "ok", res
    expected = {i: [100 * i + j for j in range(i + 1)] for i in range(5)}
    assert res[0][1] == expected and res[1][1] is None
    # one process gives the same gather and digest
    single = pd.gather_token_ids([expected[i] for i in range(5)], 5, 8)
    assert single == expected
    assert pd.tokens_digest(single) == pd.tokens_digest(res[0][1])
    assert pd.tokens_digest({0: [1]}) != pd.tokens_digest({0: [1, 2]})
