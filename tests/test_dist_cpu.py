"""Multi-rank host logic on CPU (gloo, world_size 2): batch sharding, the
cross-GPU split-KV exchange protocol (partials -> all-gather -> merge) and
failure detection when a peer rank dies.  The CUDA decode and combine are
stood in by the CPU oracle here; the same protocol runs with the CUDA
operator over NCCL in the GPU tests and the bench."""
import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _paths():
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "flashatte-hand_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _oracle_decode(q, k, v, sl, bt, scale, out_o, out_l):
    from oracle.decode_ref import decode_reference
    o, l = decode_reference(q, k, v, sl, bt, softmax_scale=scale)
    out_o.copy_(o)
    out_l.copy_(l)


def _oracle_combine(part_o, part_l, out_dtype):
    from oracle.decode_ref import merge_partials
    o, l = merge_partials(part_o, part_l)
    return o.to(out_dtype), l.float()


def _worker(rank, port, kind, errq):
    try:
        _paths()
        from flashdecode import cases, dist as fdist
        from oracle.decode_ref import decode_reference
        _init(rank, port, timeout_s=10 if kind == "peer_dies" else 60)
        case = cases.custom_case("d", torch.bfloat16, [1000, 1, 0, 2500, 300, 777], 16, 4,
                                 page=16, seed=3)
        full = cases.materialize(case, "cpu", seed=3)
        ref_o, ref_l = decode_reference(full["q"], full["k_cache"], full["v_cache"],
                                        full["cache_seqlens"], full["block_table"])
        if kind == "batch":
            sub, rows = fdist.batch_shard(case, rank, WORLD)
            # local pool = the global pages this rank owns, remapped
            used = case.block_table[rows][case.block_table[rows] >= 0].unique(sorted=True).long()
            k, v = full["k_cache"][used], full["v_cache"][used]
            o, l = decode_reference(full["q"][rows], k, v, sub.seqlens, sub.block_table)
            assert torch.allclose(o, ref_o[rows], atol=1e-6)
            got = [None] * WORLD
            dist.all_gather_object(got, rows)
            assert sorted(sum(got, [])) == list(range(case.B))
        elif kind == "splitkv":
            local, page_map = fdist.kv_split_case(case, rank, WORLD)
            k, v = full["k_cache"][page_map], full["v_cache"][page_map]
            step = fdist.SplitKVDecode(case.B, case.Hq, case.D, torch.float32, "cpu",
                                       decode_fn=_oracle_decode, combine_fn=_oracle_combine)
            out, lse = step(full["q"], k, v, local.seqlens, local.block_table, case.softmax_scale)
            assert torch.allclose(out, ref_o, atol=1e-5), float((out - ref_o).abs().max())
            fin = torch.isfinite(ref_l)
            assert torch.equal(fin, torch.isfinite(lse))
            assert torch.allclose(lse[fin], ref_l[fin], atol=1e-5)
        elif kind == "peer_dies":
            if rank == 1:
                os._exit(0)  # leaves between steps, before its collective
            local, page_map = fdist.kv_split_case(case, rank, WORLD)
            k, v = full["k_cache"][page_map], full["v_cache"][page_map]
            step = fdist.SplitKVDecode(case.B, case.Hq, case.D, torch.float32, "cpu",
                                       decode_fn=_oracle_decode, combine_fn=_oracle_combine)
            try:
                step(full["q"], k, v, local.seqlens, local.block_table, case.softmax_scale)
                res = ("not detected", "")
            except Exception as e:  # the collective ends with an error instead of hanging
                res = ("detected", type(e).__name__)
            errq.put(res)
            errq.close()
            errq.join_thread()  # flush before the hard exit below
            os._exit(0)
        dist.barrier()
        dist.destroy_process_group()
        errq.put(("ok", rank))
    except Exception:
        errq.put(("error", traceback.format_exc()))


def _run(kind, expect):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, kind, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(expect)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_batch_sharding_two_ranks():
    res = _run("batch", WORLD)
    assert all(r[0] == "ok" for r in res), res


def test_split_kv_exchange_two_ranks():
    res = _run("splitkv", WORLD)
    assert all(r[0] == "ok" for r in res), res


def test_peer_death_is_detected_not_hung():
    res = _run("peer_dies", 1)
    assert res[0][0] == "detected", res
