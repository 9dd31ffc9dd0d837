"""Worker of test_gpu_peer_exchange (one process per GPU, launched by torch.distributed.run):
the NVLink peer all-gather against NCCL's all_gather, then the sharded decode step with
both exchanges, outputs compared bit for bit."""
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
from deepseekrpc_b200.sharded import PeerExchange, ShardPlan, ShardedDecoder, all_gather, make_shard_inputs  # noqa: E402
from deepseekrpc_b200.workloads import small_config  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        # 1. exchanges of several sizes, repeated (the arrival counters only grow)
        for shape, dtype, chunks in (((2, 3, 256), torch.int32, None), ((70000,), torch.float32, 5)):
            x = PeerExchange(shape, dtype, dev, chunks=chunks)
            gen = torch.Generator(device=dev).manual_seed(100 + rank)
            for it in range(4):
                payload = (torch.randint(-2**31, 2**31 - 1, shape, generator=gen, device=dev, dtype=torch.int64)
                           .to(torch.int32).view(dtype))
                got = x.all_gather(payload).clone()
                want = all_gather(payload).view((world,) + tuple(shape))
                assert torch.equal(got.view(torch.int32), want.view(torch.int32)), f"exchange {shape} round {it}"
            torch.cuda.synchronize()
            assert int(x.err.item()) == 0
            x.close()
        # 2. the sharded step: peer exchange == NCCL exchange, bit for bit
        cfg = small_config("cfg5", context=262144)
        plan = ShardPlan(world, rank, tuple([cfg.context] * cfg.batch))
        inputs = make_shard_inputs(cfg, plan, dev)
        ref = ShardedDecoder(plan, cfg.heads, cfg.idx_heads, cfg.topk, cfg.scale, inputs["sink"], dev)
        out_nccl = ref.step(inputs).clone()
        peer = ShardedDecoder(plan, cfg.heads, cfg.idx_heads, cfg.topk, cfg.scale, inputs["sink"], dev)
        peer.use_peer_exchange()
        for _ in range(3):
            out_peer = peer.step(inputs).clone()
        torch.cuda.synchronize()
        assert int(ref.err.item()) == 0 and int(peer.err.item()) == 0 and peer.exchange_status() == 0
        assert torch.equal(ref.ids, peer.ids), "merged top-k differs between exchanges"
        assert torch.equal(out_nccl, out_peer), "attention output differs between exchanges"
        peer.close()
        if rank == 0:
            print("PEER_EXCHANGE_OK")
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
