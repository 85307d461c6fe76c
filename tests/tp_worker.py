"""Worker for the tensor-parallel parity test, one process per GPU (torchrun).

Every rank builds the same tiny model sharded over the group and checks, against the
CPU oracle, prefill logits, decode logits, 32 greedy and 16 top-p-sampled tokens -- bit
for bit.  Exit status 0 on success.  Run by tests/test_tp_gpu.py as ``tp_worker.py <flag file>``.

A rank that fails creates the flag file, aborts its communicator and exits at once; a
watchdog thread on every rank aborts the communicator and exits when the flag appears
or the deadline passes, so no rank stays in a collective waiting for a dead peer."""
import datetime
import os
import sys
import threading
import time
import traceback

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


DEADLINE_S = 180.0


def watchdog(flag, state):
    t0 = time.monotonic()
    while True:
        time.sleep(0.2)
        if os.path.exists(flag) or time.monotonic() - t0 > DEADLINE_S:
            print(f"rank {state['rank']}: peer failed or deadline passed; aborting", flush=True)
            if state.get("tp") is not None:
                state["tp"].abort()
            os._exit(3)


def main(state):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    state["rank"] = rank
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    from asicfortranai_b200.quantized import Context
    from asicfortranai_b200.tp import TPGroup
    from oracle import oracle as orc
    from tests.model_util import TINY, gpu_model, make_weights

    ctx = Context(int(os.environ["LOCAL_RANK"]))
    tp = TPGroup.from_torch(ctx, dist, timeout_s=60)
    state["tp"] = tp
    ok = True
    # the fused exchange of a row-parallel projection: x += dequant(sum over ranks of C);
    # the last case exceeds the peer-memory size and goes through NCCL
    from asicfortranai_b200 import _lib
    for rows, N in ((1, 1024), (16, 1024), (5, 2048), (64, 8192)):
        rng = np.random.default_rng(100 + rows)
        Cs = [rng.integers(-2**20, 2**20, size=(rows, N), dtype=np.int32) for _ in range(world)]
        sc = rng.random(N, dtype=np.float32) * np.float32(1e-3)
        off = rng.standard_normal(N).astype(np.float32)
        x0 = rng.standard_normal((rows, N)).astype(np.float32)
        tot = sum(c.astype(np.int64) for c in Cs).astype(np.int32)
        want = x0 + (tot.astype(np.float32) + off) * sc
        dC = torch.from_numpy(Cs[rank]).cuda()
        dx = torch.from_numpy(x0).cuda()
        ds, do = torch.from_numpy(sc).cuda(), torch.from_numpy(off).cuda()
        e_ok = True
        for rep in range(3):   # repeated calls walk the epoch parities
            dC.copy_(torch.from_numpy(Cs[rank]))
            dx.copy_(torch.from_numpy(x0))
            torch.cuda.synchronize()
            _lib.check(_lib.load().q35_tp_allreduce_dequant(tp.h, ctx.h, dC.data_ptr(), rows, N, ds.data_ptr(),
                                                             do.data_ptr(), dx.data_ptr()), "tp_allreduce_dequant")
            ctx.synchronize()
            e_ok &= np.array_equal(dx.cpu().numpy().view(np.uint32), want.view(np.uint32))
        ok &= e_ok
        print(f"rank {rank}: exchange rows {rows} N {N} bit-exact={e_ok}", flush=True)
    ctx.device_error()
    for wformat, rope_mode in ((0, 0), (1, 1)):
        kvh = max(4, world)   # every rank holds at least one KV head
        cfg = dict(TINY, n_heads=2 * kvh, n_kv_heads=kvh, hidden=256 * kvh, ffn=512 * kvh, vocab=1024,
                   wformat=wformat, rope_mode=rope_mode)
        w = make_weights(cfg, seed=11)
        om = orc.OracleModel(cfg, w)
        gm = gpu_model(ctx, cfg, w, tp)
        ids = orc.gen_tokens(9, 11, 4, cfg["vocab"])
        ref, got = om.forward(ids), gm.forward_llama(ids)
        f_ok = np.array_equal(ref.view(np.uint32), got.view(np.uint32))
        nxt, lg = gm.decode_step(want_logits=True)
        ref1 = om.forward(np.array([orc.sample_greedy(ref[-1])], np.int32))
        d_ok = np.array_equal(ref1.view(np.uint32), lg.view(np.uint32)) and nxt[0] == orc.sample_greedy(ref1[-1])
        om2 = orc.OracleModel(cfg, w)
        g_ok = np.array_equal(gm.generate(ids[None, :], 32)[0], om2.generate(ids, 32))
        # top-p sampling over the all-gathered vocabulary shards: every rank draws the
        # oracle's token from the same logits
        gm.set_sampling("top_p", top_p=0.9, seed=5)
        om3 = orc.OracleModel(cfg, w)
        s_ok = np.array_equal(gm.generate(ids[None, :], 16)[0],
                              om3.generate(ids, 16, sampling=dict(mode=3, top_p=0.9, seed=5), seq=0))
        gm.cleanup_llama_model()
        ok &= f_ok and d_ok and g_ok and s_ok
        print(f"rank {rank}: format {wformat} rope {rope_mode} forward={f_ok} decode={d_ok} "
              f"generate={g_ok} sampled={s_ok}", flush=True)
    bad = torch.tensor([0 if ok else 1])
    dist.all_reduce(bad)
    ctx.close()
    dist.destroy_process_group()
    return 1 if int(bad.item()) else 0


if __name__ == "__main__":
    flag_path = sys.argv[1]
    st = {"rank": os.environ.get("RANK"), "tp": None}
    threading.Thread(target=watchdog, args=(flag_path, st), daemon=True).start()
    try:
        code = main(st)
    except BaseException:
        traceback.print_exc()
        sys.stdout.flush()
        sys.stderr.flush()
        open(flag_path, "w").close()
        if st.get("tp") is not None:
            st["tp"].abort()
        os._exit(2)
    os._exit(code)
