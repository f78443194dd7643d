"""Split-KV decode across the GPUs of one box, checked against the oracle.

Run under torch.distributed.run, one rank per GPU:
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P tests/splitkv_worker.py

Every rank builds its shard of the same seeded caches (positions
shard_range(ctx, N, rank) of every sequence), runs the RoPE + owner
cache-write + split-KV attention + record exchange + merge through the C ABI
(tg_decode_layer_splitkv) and compares the replicated output with the CPU
oracle, under the automatic exchange (peer memory for the bf16 cache when
the GPUs map each other's memory) and the NCCL all-gather.  The layer from
the normed hidden state (tg_decode_layer_splitkv_x: Q/K/V projection, then
split-KV attention) is checked against the same layer on one GPU over the
whole cache.  Batched calls with page-locked buffers (three layers per batch,
position sets alternating over the same staging slots) and sequence-partitioned
decode (each rank its own sequences, no collective) are checked against the
oracle too.  Exit status 0 on success on every rank.
"""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))


def main() -> int:
    import torch
    import torch.distributed as dist
    from conftest import load_package
    import cases

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    tg = load_package()
    be = tg.CudaBackend(local)
    uid = [tg.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    be.comm_init(uid[0], rank, world, timeout_ms=60000)

    ok = True
    cases_run = [(ex, bf16, tol) for ex in (tg.EXCHANGE_AUTO, tg.EXCHANGE_NCCL)
                 for bf16, tol in ((True, 2e-3), (False, 1e-4))]
    for ex, bf16, tol in cases_run:
        be.set_exchange(ex)
        positions = [9000, 777, 12345, 0, world * 64]
        B = len(positions)
        gctx = max(positions) + 1
        start, length = tg.shard_range(gctx, world, rank)
        kv = tg.KVCache(be, 1, B, max(length, 1), shard_start=start, global_ctx=gctx,
                        dtype=tg.DTYPE_BF16 if bf16 else tg.DTYPE_F32)
        Q = np.zeros((B, cases.QD), np.float32)
        K = np.zeros((B, cases.KD), np.float32)
        V = np.zeros((B, cases.KD), np.float32)
        refs = []
        for i, p in enumerate(positions):
            q, k_new, v_new, kc, vc = cases.decode_inputs(77, p, bf16, seq=i)
            lo, hi = start, min(start + length, p)      # rows before the new token
            if hi > lo:
                kv.write_rows(0, i, 0, kc[lo:hi], vc[lo:hi])
            Q[i], K[i], V[i] = q, k_new, v_new
            refs.append(cases.oracle_decode(77, p, bf16, seq=i))
        # Three steps from the same inputs: the peer-memory exchange
        # alternates its receive buffers and flags between launches.
        for it in range(3):
            Qi, Ki = Q.copy(), K.copy()
            out = np.zeros((B, cases.QD), np.float32)
            kv.decode_layer_splitkv(0, Qi, Ki, V, np.array(positions, np.int32), out)
            for i, p in enumerate(positions):
                qr, kr, _, kc, vc, ctx = refs[i]
                err = float(np.abs(out[i] - ctx).max())
                same_q = np.array_equal(Qi[i].view(np.uint32), qr.view(np.uint32))
                if err > tol or not same_q:
                    print(f"rank {rank}: step {it} seq {i} pos {p} bf16={bf16} err={err} "
                          f"rope_ok={same_q}")
                    ok = False
                if start <= p < start + length:          # this rank owns the new row
                    krow, _ = kv.read_rows(0, i, p - start, 1)
                    want = cases.O.pack_bf16(kc[p]) if bf16 else kc[p]
                    if not np.array_equal(krow[0], want):
                        print(f"rank {rank}: cache-write mismatch seq {i}")
                        ok = False
        used = be.exchange
        if rank == 0:
            print(f"exchange requested {ex} used {used} bf16={bf16}")
        if ex == tg.EXCHANGE_NCCL and used != tg.EXCHANGE_NCCL:
            print(f"rank {rank}: NCCL exchange requested, {used} used")
            ok = False
        if not bf16 and used == tg.EXCHANGE_PEER:
            print(f"rank {rank}: fp32 cache cannot use the peer exchange")
            ok = False
        # all ranks hold the same output
        t = torch.from_numpy(out.copy())
        gathered = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        if not all(torch.equal(gathered[0], g) for g in gathered):
            print(f"rank {rank}: outputs differ across ranks")
            ok = False
        kv.destroy()
    # BASELINE config 4 at full size: 4 sequences at position 131071 (131072
    # rows each, bf16), the rows sharded over the world, one layer, three
    # steps per exchange and decode ring, against the oracle's decode step
    # (tmac_gguf.cpp:990-1016 / :1090-1128 restated) on the same values.
    ctx4, B4 = 131072, 4
    pos4 = np.full(B4, ctx4 - 1, np.int32)
    start, length = tg.shard_range(ctx4, world, rank)
    kv = tg.KVCache(be, 1, B4, length, shard_start=start, global_ctx=ctx4, dtype=tg.DTYPE_BF16)
    Q = np.zeros((B4, cases.QD), np.float32)
    K = np.zeros((B4, cases.KD), np.float32)
    V = np.zeros((B4, cases.KD), np.float32)
    ref4 = []
    for i in range(B4):
        qr, kr, _, kc, vc, ctx = cases.oracle_decode(91, ctx4 - 1, True, seq=i)
        q, k_new, v_new, _, _ = cases.decode_inputs(91, ctx4 - 1, True, seq=i)
        hi = min(start + length, ctx4 - 1)
        if hi > start:
            kv.write_rows(0, i, 0, kc[start:hi], vc[start:hi])
        Q[i], K[i], V[i] = q, k_new, v_new
        ref4.append((qr, ctx))
        del kc, vc
    for ex in (tg.EXCHANGE_AUTO, tg.EXCHANGE_NCCL):
        be.set_exchange(ex)
        for ring, pre in ((0, 0), (128, 1), (192, 1)):
            tg.set_decode_tuning(ring, pre)
            for it in range(3):
                Qi, Ki = Q.copy(), K.copy()
                out = np.zeros((B4, cases.QD), np.float32)
                kv.decode_layer_splitkv(0, Qi, Ki, V, pos4, out)
                for i in range(B4):
                    err = float(np.abs(out[i] - ref4[i][1]).max())
                    same_q = np.array_equal(Qi[i].view(np.uint32), ref4[i][0].view(np.uint32))
                    if err > 2e-3 or not same_q:
                        print(f"rank {rank}: config 4 exchange {ex} ring {ring} preload {pre} "
                              f"step {it} seq {i} err={err} rope_ok={same_q}")
                        ok = False
        if rank == 0:
            print(f"config 4 x{world}: exchange requested {ex} used {be.exchange}, "
                  f"max err {max(float(np.abs(out[i] - ref4[i][1]).max()) for i in range(B4)):.2e}")
    tg.set_decode_tuning(0, 0)
    kv.destroy()
    # The layer from the normed hidden state x (projection + split-KV
    # attention) against the same layer on this GPU over the whole cache:
    # the owner's new k / v row is bit-identical, the output agrees to the
    # split-merge rounding.
    be.set_exchange(tg.EXCHANGE_AUTO)
    for bf16 in (True, False):
        positions = [9000, 777, 12345, 0, world * 64]
        B = len(positions)
        gctx = max(positions) + 1
        start, length = tg.shard_range(gctx, world, rank)
        dt = tg.DTYPE_BF16 if bf16 else tg.DTYPE_F32
        kv = tg.KVCache(be, 1, B, max(length, 1), shard_start=start, global_ctx=gctx, dtype=dt)
        full = tg.KVCache(be, 1, B, gctx, dtype=dt)
        for i, p in enumerate(positions):
            _, _, _, kc, vc = cases.decode_inputs(78, p, bf16, seq=i)
            lo, hi = start, min(start + length, p)
            if hi > lo:
                kv.write_rows(0, i, 0, kc[lo:hi], vc[lo:hi])
            if p > 0:
                full.write_rows(0, i, 0, kc[:p], vc[:p])
        wq, wk, wv, bq, bk, bv = cases.qkv_weights(79, 8, True)
        W = tg.QKVWeights(wq, wk, wv, 896, v_type=8, b_q=bq, b_k=bk, b_v=bv)
        X = cases.qkv_x(80, B).copy()
        ref = np.zeros((B, cases.QD), np.float32)
        full.decode_layer_x(0, W, X, positions, ref)
        for it in range(2):
            out = np.zeros((B, cases.QD), np.float32)
            kv.decode_layer_splitkv_x(0, W, X, positions, out)
            err = float(np.abs(out - ref).max())
            if err > 5e-5:
                print(f"rank {rank}: x path step {it} bf16={bf16} err={err}")
                ok = False
        for i, p in enumerate(positions):
            if start <= p < start + length:
                a = kv.read_rows(0, i, p - start, 1)
                b = full.read_rows(0, i, p, 1)
                if not (np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])):
                    print(f"rank {rank}: x path cache row mismatch seq {i}")
                    ok = False
        # The attention block (projection, split attention, attn_output +
        # residual on every rank) against the one-GPU block.
        wo = cases.attn_output_weight(81, 6)
        h0 = cases.residual_in(82, B)
        hid = h0.copy()
        kv.attention_block(0, W, wo, X, positions, hid, o_type=6, split=True)
        full2 = tg.KVCache(be, 1, B, gctx, dtype=dt)
        for i, p in enumerate(positions):
            _, _, _, kc, vc = cases.decode_inputs(78, p, bf16, seq=i)
            if p > 0:
                full2.write_rows(0, i, 0, kc[:p], vc[:p])
        hid_ref = h0.copy()
        full2.attention_block(0, W, wo, X, positions, hid_ref, o_type=6)
        full2.destroy()
        err = float(np.abs(hid - hid_ref).max())
        if err > 2e-4:
            print(f"rank {rank}: attention block bf16={bf16} err={err}")
            ok = False
        if rank == 0:
            print(f"x path bf16={bf16} exchange {be.exchange} block err {err:.2e}")
        kv.destroy()
        full.destroy()
    # Inside a batch with page-locked host buffers, as a forward loop calls
    # the library (and bench.py's end-to-end loop): three layers per batch,
    # two position sets alternating over the same staging slots, outputs
    # reaching the host at tg_batch_end; every layer against the oracle.
    be.set_exchange(tg.EXCHANGE_AUTO)
    layers = 3
    sets = ([9000, 777, 12345, 0], [12000, 5, 640, world * 64 + 1])
    gctx = max(max(s) for s in sets) + 1
    start, length = tg.shard_range(gctx, world, rank)
    kvs, data = [], []
    for j, positions in enumerate(sets):
        B = len(positions)
        kvj = tg.KVCache(be, layers, B, max(length, 1), shard_start=start, global_ctx=gctx,
                         dtype=tg.DTYPE_BF16)
        ins, refs = [], []
        for layer in range(layers):
            Q = np.zeros((B, cases.QD), np.float32)
            K = np.zeros((B, cases.KD), np.float32)
            V = np.zeros((B, cases.KD), np.float32)
            lrefs = []
            for i, p in enumerate(positions):
                q, k_new, v_new, kc, vc = cases.decode_inputs(60 + j, p, True, seq=i, layer=layer)
                hi = min(start + length, p)
                if hi > start:
                    kvj.write_rows(layer, i, 0, kc[start:hi], vc[start:hi])
                Q[i], K[i], V[i] = q, k_new, v_new
                r = cases.oracle_decode(60 + j, p, True, seq=i, layer=layer)
                lrefs.append((r[0], r[5]))
            ins.append((Q, K, V))
            refs.append(lrefs)
        kvs.append(kvj)
        data.append((torch.from_numpy(np.array(positions, np.int32)).pin_memory(), ins, refs))
    worst = 0.0
    for rnd, j in enumerate((0, 1, 0, 1)):
        kvj, (pos_pin, ins, refs) = kvs[j], data[j]
        # Every buffer of the batch stays allocated until tg_batch_end: the
        # rotated q / k and the outputs reach the host there (a buffer freed
        # earlier may already belong to another tensor).
        res = []
        be.metal_batch_begin()
        for layer in range(layers):
            Qp, Kp, Vp = (torch.from_numpy(x.copy()).pin_memory() for x in ins[layer])
            outp = torch.zeros(Qp.shape, dtype=torch.float32).pin_memory()
            kvj.decode_layer_splitkv(layer, Qp, Kp, Vp, pos_pin, outp)
            res.append((Qp, Kp, Vp, outp))
        be.metal_batch_end()
        for layer in range(layers):
            qo, o = res[layer][0].numpy(), res[layer][3].numpy()
            for i, p in enumerate(sets[j]):
                qr, ctx = refs[layer][i]
                err = float(np.abs(o[i] - ctx).max())
                worst = max(worst, err)
                same_q = np.array_equal(qo[i].view(np.uint32), qr.view(np.uint32))
                if err > 2e-3 or not same_q:
                    print(f"rank {rank}: batched round {rnd} layer {layer} seq {i} pos {p} "
                          f"err={err} rope_ok={same_q}")
                    ok = False
    if rank == 0:
        print(f"batched page-locked split-KV x{world}: exchange {be.exchange}, "
              f"max err {worst:.2e}")
    for kvj in kvs:
        kvj.destroy()
    # Sequence-partitioned decode (BASELINE configs 2-3 over several GPUs):
    # rank r owns sequences r, r + world, ... of one ragged batch and their
    # caches, with no collective on the data path; bf16 and fp32 caches
    # against the oracle.
    glob = [3, 70, 1025, 4000, 9000, 64, 511, 2049]
    mine = list(range(rank, len(glob), world))
    for bf16, tol in ((True, 2e-3), (False, 1e-4)):
        pr = [glob[s] for s in mine]
        kvp = tg.KVCache(be, 1, len(pr), max(pr) + 1,
                         dtype=tg.DTYPE_BF16 if bf16 else tg.DTYPE_F32)
        Q = np.zeros((len(pr), cases.QD), np.float32)
        K = np.zeros((len(pr), cases.KD), np.float32)
        V = np.zeros((len(pr), cases.KD), np.float32)
        refs = []
        for i, s in enumerate(mine):
            p = glob[s]
            q, k_new, v_new, kc, vc = cases.decode_inputs(66, p, bf16, seq=s)
            if p > 0:
                kvp.write_rows(0, i, 0, kc[:p], vc[:p])
            Q[i], K[i], V[i] = q, k_new, v_new
            refs.append(cases.oracle_decode(66, p, bf16, seq=s)[5])
        out = np.zeros((len(pr), cases.QD), np.float32)
        kvp.decode_layer(0, Q, K, V, np.array(pr, np.int32), out)
        for i, s in enumerate(mine):
            err = float(np.abs(out[i] - refs[i]).max())
            if err > tol:
                print(f"rank {rank}: sequence-partitioned seq {s} bf16={bf16} err={err}")
                ok = False
        kvp.destroy()
    if rank == 0:
        print(f"sequence-partitioned x{world}: {len(glob)} sequences checked")
    # Failure detection: with a 1 s wait limit, rank 1 skips one layer's
    # call (it stays alive, its memory stays mapped, nothing of it is in
    # flight).  Every other rank's merge kernel stops waiting for rank 1's
    # records and the call reports TG_ERR_DEVICE (device error 0x105) at its
    # synchronisation.  All ranks then destroy and re-create the
    # communicator, and the next step matches the oracle again.
    be.set_exchange(tg.EXCHANGE_AUTO)
    be.set_wait_limit_ms(1000)
    positions = [5000, 77, world * 64 + 3]
    B = len(positions)
    gctx = max(positions) + 1
    start, length = tg.shard_range(gctx, world, rank)
    kv = tg.KVCache(be, 1, B, max(length, 1), shard_start=start, global_ctx=gctx,
                    dtype=tg.DTYPE_BF16)
    Q = np.zeros((B, cases.QD), np.float32)
    K = np.zeros((B, cases.KD), np.float32)
    V = np.zeros((B, cases.KD), np.float32)
    refs = []
    for i, p in enumerate(positions):
        q, k_new, v_new, kc, vc = cases.decode_inputs(55, p, True, seq=i)
        hi = min(start + length, p)
        if hi > start:
            kv.write_rows(0, i, 0, kc[start:hi], vc[start:hi])
        Q[i], K[i], V[i] = q, k_new, v_new
        refs.append(cases.oracle_decode(55, p, True, seq=i)[5])

    def run_step():
        out = np.zeros((B, cases.QD), np.float32)
        kv.decode_layer_splitkv(0, Q.copy(), K.copy(), V, np.array(positions, np.int32), out)
        return max(float(np.abs(out[i] - refs[i]).max()) for i in range(B))

    err0 = run_step()                      # all ranks: a good step first
    if err0 > 2e-3:
        print(f"rank {rank}: pre-failure step err={err0}")
        ok = False
    dist.barrier()
    import time
    if rank != 1:
        t0 = time.perf_counter()
        try:
            run_step()
            print(f"rank {rank}: a step without rank 1 did not fail")
            ok = False
        except tg.TGError as e:
            dt = time.perf_counter() - t0
            if e.status != tg.TG_ERR_DEVICE or "0x105" not in e.message or dt > 30:
                print(f"rank {rank}: unexpected failure {e.status} {e.message} after {dt:.1f} s")
                ok = False
            elif rank == 0:
                print(f"failure detected in {dt:.2f} s: {e.message}")
    dist.barrier()                         # rank 1 waited here, idle, memory mapped
    be.comm_destroy()
    uid = [tg.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    be.comm_init(uid[0], rank, world, timeout_ms=60000)
    be.set_wait_limit_ms(5000)
    kv.destroy()
    kv = tg.KVCache(be, 1, B, max(length, 1), shard_start=start, global_ctx=gctx,
                    dtype=tg.DTYPE_BF16)
    for i, p in enumerate(positions):
        _, _, _, kc, vc = cases.decode_inputs(55, p, True, seq=i)
        hi = min(start + length, p)
        if hi > start:
            kv.write_rows(0, i, 0, kc[start:hi], vc[start:hi])
    err1 = run_step()
    if err1 > 2e-3 or be.exchange != tg.EXCHANGE_PEER:
        print(f"rank {rank}: after recovery err={err1} exchange={be.exchange}")
        ok = False
    elif rank == 0:
        print(f"recovered: step err {err1:.2e} over the re-created communicator")
    kv.destroy()
    be.comm_destroy()
    be.shutdown()
    flag = torch.tensor([1 if ok else 0])
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0:
        print("splitkv worker:", "PASS" if flag.item() == 1 else "FAIL", f"world={world}")
    return 0 if flag.item() == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
