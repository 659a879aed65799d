"""Sharding of independent streams over ranks (whisper4j_b200/shard.py), on CPU with gloo.

Streams are the reference's independent 30 s chunks (WhisperModel.java:334-430).  The ranks run
the oracle's greedy decode on their share; rank 0's gathered results must equal one process
decoding every stream.  A failing rank must end the others with an error, not a hang.
"""
import datetime
import multiprocessing as mp
import os
import socket

import pytest

from whisper4j_b200.shard import shard_streams

N_STREAMS, MAX_TOKENS = 5, 6


def test_round_robin_partition():
    for world in (1, 2, 3, 8):
        parts = [shard_streams(11, world, r) for r in range(world)]
        assert sorted(i for p in parts for i in p) == list(range(11))
        for r, p in enumerate(parts):
            assert all(i % world == r for i in p)
    assert shard_streams(0, 4, 3) == []
    with pytest.raises(ValueError):
        shard_streams(4, 2, 2)


def _decode(indices):
    from oracle import oracle as O

    from .helpers import SMALL, SMALL_OPTS, encoder_output, parsed

    m = O.OracleModel(parsed(SMALL, 5, "f16", tuple(sorted(SMALL_OPTS.items()))))
    out = []
    for i in indices:
        xa = encoder_output(100 + i, SMALL.n_audio_ctx, SMALL.n_text_state)
        r = m.decode(xa, [996, 997, 998, 999], 999, MAX_TOKENS, suppress=[999])
        out.append((i, r["tokens"], round(r["sum_logprob"], 9)))
    return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, fail_rank, q):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist

    from whisper4j_b200.shard import decode_sharded

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        def dec(idx):
            if rank == fail_rank:
                raise RuntimeError("injected failure on the host")
            return _decode(idx)

        res = decode_sharded(N_STREAMS, dec)
        q.put((rank, "ok", res))
    except Exception as e:  # the failing rank, or a peer whose gather ran out of time
        q.put((rank, "error", type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, status, payload = q.get(timeout=120)
        out[rank] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_two_ranks_gather_equals_single_process():
    out = _run(2)
    assert out[0][0] == "ok" and out[1] == ("ok", None)
    assert out[0][1] == _decode(range(N_STREAMS))


def test_failing_rank_ends_the_others_with_an_error():
    out = _run(2, fail_rank=1)
    assert out[1] == ("error", "RuntimeError")
    assert out[0][0] == "error"
