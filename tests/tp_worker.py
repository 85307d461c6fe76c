"""Worker for the tensor-parallel parity test, one process per GPU (torchrun).

Every rank builds the same tiny model sharded over the group and checks, against the
CPU oracle, prefill logits, decode logits and 32 greedy tokens -- bit for bit.  Exit
status 0 on success.  Run by tests/test_tp_gpu.py."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    from asicfortranai_b200.quantized import Context
    from asicfortranai_b200.tp import TPGroup
    from oracle import oracle as orc
    from tests.model_util import TINY, gpu_model, make_weights

    ctx = Context(int(os.environ["LOCAL_RANK"]))
    tp = TPGroup.from_torch(ctx, dist, timeout_s=60)
    ok = True
    for wformat, rope_mode in ((0, 0), (1, 1)):
        cfg = dict(TINY, n_heads=8, n_kv_heads=4, hidden=1024, ffn=2048, vocab=1024,
                   wformat=wformat, rope_mode=rope_mode)
        w = make_weights(cfg, seed=11)
        om = orc.OracleModel(cfg, w)
        gm = gpu_model(ctx, cfg, w, tp)
        ids = orc.gen_tokens(9, 11, 4, cfg["vocab"])
        ref, got = om.forward(ids), gm.forward_llama(ids)
        ok &= np.array_equal(ref.view(np.uint32), got.view(np.uint32))
        nxt, lg = gm.decode_step(want_logits=True)
        ref1 = om.forward(np.array([orc.sample_greedy(ref[-1])], np.int32))
        ok &= np.array_equal(ref1.view(np.uint32), lg.view(np.uint32))
        om2 = orc.OracleModel(cfg, w)
        ok &= np.array_equal(gm.generate(ids[None, :], 32)[0], om2.generate(ids, 32))
        gm.cleanup_llama_model()
        print(f"rank {rank}: format {wformat} rope {rope_mode} bit-exact={ok}", flush=True)
    flag = torch.tensor([0 if ok else 1])
    dist.all_reduce(flag)
    tp.close()
    ctx.close()
    dist.destroy_process_group()
    sys.exit(1 if int(flag.item()) else 0)


if __name__ == "__main__":
    main()
