"""Host-side logic of the multi-GPU paths on CPU ranks (gloo, world size 2).

The CUDA partial / merge functions are replaced by the oracle's CPU versions, so these
tests exercise the page windows, the all-gather of (O, LSE) partials, the merge and the
failure behaviour of a rank that dies before the collective -- no GPU involved."""

from __future__ import annotations

import datetime
import os
import socket
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    rng = np.random.default_rng(42)
    q = rng.standard_normal((2, 8, 64)).astype(np.float32)
    k = rng.standard_normal((2, 8, 300, 64)).astype(np.float32)
    v = rng.standard_normal((2, 8, 300, 64)).astype(np.float32)
    lengths = np.array([300, 170])
    return q, k, v, lengths


def _worker(rank, world, port, out_dir, mode):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "oracle"))
    import flashspec_oracle as O

    from flashspec_b200.dist import SequenceShardedDecoder

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    q, k, v, lengths = _data()

    def partial(qt, cache, window):
        lo, hi = window
        o, lse = O.partial_attention(q, k, v, lo * 16, hi * 16, lengths)
        return torch.from_numpy(o), torch.from_numpy(lse)

    def merge(o_parts, lse_parts, dtype):
        return torch.from_numpy(O.merge_partials(o_parts.numpy(), lse_parts.numpy())).to(dtype)

    dec = SequenceShardedDecoder(partial_fn=partial, merge_fn=merge)
    result = "ok"
    try:
        if mode == "die" and rank == 1:
            raise SystemExit(3)  # this rank leaves before the collective
        out = dec(torch.from_numpy(q), None, n_pages=(300 + 15) // 16, out_dtype=torch.float32)
        ref = O.reference_attention(q, k, v, lengths)
        np.testing.assert_allclose(out.numpy(), ref, atol=2e-6, rtol=1e-5)
        lo, hi = dec.window(19)
        result = f"ok {lo} {hi}"
    except SystemExit:
        raise
    except Exception as exc:  # noqa: BLE001 - the failure is the result we record
        result = f"error {type(exc).__name__}"
    (Path(out_dir) / f"rank{rank}.txt").write_text(result)
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def _run(mode):
    port = _free_port()
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_worker, args=(r, 2, port, d, mode)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
        return [(Path(d) / f"rank{r}.txt").read_text() if (Path(d) / f"rank{r}.txt").exists() else None
                for r in range(2)], [p.exitcode for p in procs]


def test_sequence_sharded_merge_equals_full_attention():
    res, codes = _run("ok")
    assert codes == [0, 0]
    assert res[0] == "ok 0 9" and res[1] == "ok 9 19"


def test_rank_that_leaves_before_the_collective_is_detected():
    res, codes = _run("die")
    assert codes[1] == 3
    assert res[0] is not None and res[0].startswith("error")


def test_page_window_and_request_shard():
    from flashspec_b200.dist import page_window, request_shard

    spans = [page_window(8192, r, 8) for r in range(8)]
    assert spans[0] == (0, 1024) and spans[-1] == (7168, 8192)
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert page_window(5, 1, 2) == (2, 5)
    with pytest.raises(ValueError):
        page_window(10, 2, 2)
    lens = [8192 - 128 * i for i in range(64)]
    shards = request_shard(lens, 4)
    assert sorted(i for s in shards for i in s) == list(range(64))
    loads = [sum(lens[i] for i in s) for s in shards]
    assert max(loads) - min(loads) <= max(lens)
