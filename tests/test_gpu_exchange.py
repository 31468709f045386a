"""The fused Ulysses exchange (pasa_b200.exchange: q/k/v producer and PASA
epilogue storing into the other GPUs' buffers) on 2 GPUs: the DiT step is
bit-identical to the step with NCCL all-to-alls, and matches the 1-GPU step.
Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    from pasa_b200 import dit
    return dit.DiTConfig(hidden=512, heads=4, ffn=1024, layers=2, text_len=16, frames=2, height=16, width=32,
                         in_channels=16, text_dim=64, freq_dim=32, density=0.25)


def _inputs(cfg, device):
    from pasa_b200 import dit
    g = torch.Generator().manual_seed(5)
    lat = torch.randn((1, cfg.in_channels, cfg.frames, 2 * cfg.height, 2 * cfg.width), generator=g)
    txt = torch.randn((1, cfg.text_len, cfg.text_dim), generator=g)
    blocks = [dit.init_block(cfg, 30 + i, device) for i in range(cfg.layers)]
    emb = dit.init_embed(cfg, 3, device)
    return dit.patchify(lat).to(torch.bfloat16).to(device), txt.to(torch.bfloat16).to(device), blocks, emb


def _worker(rank, port, q):
    import datetime

    import torch.distributed as dist

    from pasa_b200 import dit
    from pasa_b200.exchange import UlyssesPeerExchange

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    ex = None
    try:
        cfg = _cfg()
        lat, txt, blocks, emb = _inputs(cfg, dev)
        t0, t1 = dit.local_slice(cfg, rank, WORLD)
        cos, sin = dit.rope_table(cfg, dev)
        rope = (cos[t0:t1].contiguous(), sin[t0:t1].contiguous())
        t = torch.tensor([700], device=dev)
        core = dit.pasa_core(cfg.density)
        ex = UlyssesPeerExchange(dist.group.WORLD, dev, cfg.heads, cfg.head_dim, t1 - t0)
        with torch.no_grad():
            a = dit.step(lat[:, t0:t1], t, txt, rope, emb, blocks, cfg, core, dist.group.WORLD, fused=True,
                         exchange=ex)
            b = dit.step(lat[:, t0:t1], t, txt, rope, emb, blocks, cfg, core, dist.group.WORLD, fused=True)
            a2 = dit.step(lat[:, t0:t1], t, txt, rope, emb, blocks, cfg, core, dist.group.WORLD, fused=True,
                          exchange=ex)                       # buffers reused: still the same
        torch.cuda.synchronize()
        q.put((rank, torch.equal(a, b), torch.equal(a, a2), a.float().cpu()))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))
        raise
    finally:
        if ex is not None:
            ex.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_peer_exchange_equals_all_to_all_and_single_gpu():
    import torch.multiprocessing as mp

    from pasa_b200 import dit
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=300) for _ in range(WORLD)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    assert all(len(r) == 4 for r in results), results
    assert all(r[1] for r in results), "peer exchange differs from the NCCL all-to-all"
    assert all(r[2] for r in results), "second step through the same buffers differs"
    assert all(p.exitcode == 0 for p in procs)
    # against the whole step on one GPU (GEMMs on other row counts: tolerance)
    cfg = _cfg()
    dev = torch.device("cuda", 0)
    lat, txt, blocks, emb = _inputs(cfg, dev)
    with torch.no_grad():
        one = dit.step(lat, torch.tensor([700], device=dev), txt, dit.rope_table(cfg, dev), emb, blocks, cfg,
                       dit.pasa_core(cfg.density), fused=True).float().cpu()
    got = torch.cat([r[3] for r in results], dim=1)
    assert torch.nn.functional.cosine_similarity(got.flatten(), one.flatten(), dim=0).item() > 0.9999
    assert (got - one).abs().max().item() < 2e-2 * one.abs().max().item()
