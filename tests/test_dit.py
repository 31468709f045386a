"""The DiT denoising step (pasa_b200.dit) on CPU: patch layout, and the
Ulysses sequence<->head resharding over gloo ranks (world size 2 and 4) giving
the single-process step's output with an exact fp32 attention core."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from pasa_b200 import dit

CFG = dit.DiTConfig(hidden=64, heads=4, ffn=128, layers=2, text_len=8, frames=2, height=4, width=4,
                    in_channels=4, text_dim=32, freq_dim=16)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(cfg):
    g = torch.Generator().manual_seed(0)
    lat = torch.randn((1, cfg.in_channels, cfg.frames, 2 * cfg.height, 2 * cfg.width), generator=g)
    txt = torch.randn((1, cfg.text_len, cfg.text_dim), generator=g)
    blocks = [dit.init_block(cfg, 10 + i, "cpu", torch.float32) for i in range(cfg.layers)]
    emb = dit.init_embed(cfg, 1, "cpu", torch.float32)
    return lat, txt, blocks, emb


def _sdpa(q, k, v):
    return F.scaled_dot_product_attention(q, k, v)


def _single(cfg):
    lat, txt, blocks, emb = _inputs(cfg)
    return dit.step(dit.patchify(lat), torch.tensor([500]), txt, dit.rope_table(cfg, "cpu"), emb, blocks, cfg, _sdpa)


def test_patchify_is_the_strided_convolution():
    lat, _, _, emb = _inputs(CFG)
    p = dit.patchify(lat)
    assert torch.equal(dit.unpatchify(p, CFG), lat)
    w = emb["patch"].reshape(CFG.hidden, CFG.in_channels, 1, 2, 2)
    conv = F.conv3d(lat, w, emb["patch_b"], stride=(1, 2, 2)).flatten(2).transpose(1, 2)
    assert torch.allclose(conv, F.linear(p, emb["patch"], emb["patch_b"]), atol=1e-6)


def test_rope_table_splits_the_head_dimension():
    cfg = dit.DiTConfig(frames=2, height=3, width=5)
    cos, sin = dit.rope_table(cfg, "cpu")
    assert cos.shape == (30, 64)                           # D/2 pairs: 22 frame, 21 row, 21 column
    # token (f=1, r=0, c=0): only the frame pairs rotate
    ang = torch.atan2(sin[15], cos[15])
    assert (ang[:22] != 0).all() and (ang[22:] == 0).all()
    x = torch.randn((1, 1, 30, 128))
    y = dit.apply_rope(x, cos, sin)                        # a rotation keeps every pair's norm
    assert torch.allclose(x.unflatten(-1, (-1, 2)).norm(dim=-1), y.unflatten(-1, (-1, 2)).norm(dim=-1), atol=1e-5)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = CFG
        lat, txt, blocks, emb = _inputs(cfg)
        t0, t1 = dit.local_slice(cfg, rank, world)
        cos, sin = dit.rope_table(cfg, "cpu")
        # resharding round trip on a tagged tensor
        B, H, D = 1, cfg.heads, 8
        full = torch.arange(B * H * cfg.tokens * D, dtype=torch.float32).reshape(B, H, cfg.tokens, D)
        mine = full[:, :, t0:t1].contiguous()
        hs = dit.seq_to_head(mine, dist.group.WORLD)
        hl = H // world
        ok_fwd = torch.equal(hs, full[:, rank * hl:(rank + 1) * hl])
        ok_back = torch.equal(dit.head_to_seq(hs, dist.group.WORLD), mine) and torch.equal(
            dit.head_to_tokens(hs, dist.group.WORLD), mine.transpose(1, 2).flatten(2, 3))
        out = dit.step(dit.patchify(lat)[:, t0:t1], torch.tensor([500]), txt, (cos[t0:t1], sin[t0:t1]), emb,
                       blocks, cfg, _sdpa, dist.group.WORLD)
        q.put((rank, ok_fwd, ok_back, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_step_matches_single_process(world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted((q.get(timeout=240) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r[1] and r[2] for r in results)
    got = torch.cat([r[3] for r in results], dim=1)
    want = _single(CFG)
    assert torch.allclose(got, want, atol=1e-5, rtol=1e-5), (got - want).abs().max()


def test_local_slice_rejects_ragged_split():
    with pytest.raises(ValueError):
        dit.local_slice(dit.DiTConfig(frames=1, height=3, width=3), 0, 2)
