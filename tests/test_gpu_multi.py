"""Multi-GPU paths (skipped with fewer than 2 GPUs) against the same computation on one GPU,
same weights and inputs: Ulysses sequence parallelism of the Flux2 and LTX-2 denoise loops over
NCCL and over the peer transport, the CFG branch split, and the VAE tile scatter.

Only the key order inside each attention changes (rank-major), so the results agree to fp32
summation-order noise: cosine >= 0.9999 and max relative error <= 1e-2.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs"),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _flux_case():
    from oracle import flux2 as ref
    from kinomlx_b200.flux2.config import FluxVariant
    from kinomlx_b200.synthetic import flux_weights, normal

    v = FluxVariant(dim=1024, heads=8, mlp="gelu_tanh", mlp_hidden=4096, rope_axes=(64, 64),
                    rope_theta=10000.0, in_channels=64, context_dim=256, double_blocks=2,
                    single_blocks=2)
    w = flux_weights(v, seed=42)
    nt, side = 64, 16
    noise = normal((1, side * side, v.in_channels), seed=43)
    text = normal((1, nt, v.context_dim), seed=44)
    ids = torch.cat([torch.zeros((1, nt, 2), dtype=torch.int64), ref.image_ids(side, side, 2)], 1)
    return v, w, noise, text, ids


def _ltx_case():
    from oracle import ltx2 as ref
    from kinomlx_b200.ltx2.config import LTXVariant
    from kinomlx_b200.synthetic import ltx_weights, normal

    v = LTXVariant(dim=1024, heads=8, context_dim=1024, blocks=2)
    w = ltx_weights(v, seed=7)
    grid = (2, 8, 8)
    latent = normal((1, 128, 128), seed=8)
    context = normal((1, 32, 1024), seed=9)
    pos = ref.pixel_coords(ref.patch_grid_bounds(*grid))
    return v, w, latent, context, pos


MINI_VAE = (("res", 1), ("d2s", (2, 2, 2), 2), ("res", 1), ("d2s", (1, 2, 2), 1), ("res", 1))


def _vae_case(device):
    from kinomlx_b200.ltx2 import video_vae as vae
    from kinomlx_b200.synthetic import make_weights, normal

    v = vae.VaeVariant(norm="group32", causal=True, top_width=256, blocks=MINI_VAE)
    w = make_weights(vae.vae_weight_specs(v), seed=13)
    return vae.VideoDecoder(w, v, device), normal((1, 128, 2, 7, 10), seed=14).to(device)


def _run(case: str, device, sp=None):
    if case == "vae":
        dec, latent = _vae_case(device)
        return dec.decode(latent, tile=4, overlap=1)
    if case == "cfg":
        from kinomlx_b200.flux2 import sampling
        from kinomlx_b200.flux2.transformer import Flux2Transformer
        from kinomlx_b200.synthetic import normal

        v, w, noise, text, ids = _flux_case()
        negative = normal(tuple(text.shape), seed=45)
        model = Flux2Transformer(w, v, device)
        return sampling.denoise_joint(model, noise, text, ids, sigmas=sampling.linear_sigmas(3),
                                negative=negative, guidance=4.0)
    if case == "flux":
        from kinomlx_b200.flux2 import sampling
        from kinomlx_b200.flux2.transformer import Flux2Transformer

        v, w, noise, text, ids = _flux_case()
        model = Flux2Transformer(w, v, device, sp=sp)
        return sampling.denoise_joint(model, noise, text, ids, sigmas=sampling.linear_sigmas(3))
    from kinomlx_b200.ltx2 import denoise as ldn
    from kinomlx_b200.ltx2.transformer import LTXVideoTransformer

    v, w, latent, context, pos = _ltx_case()
    model = LTXVideoTransformer(w, v, device, sp=sp)
    return ldn.denoise_video(model, latent, context, pos, sigmas=ldn.DISTILLED_STAGE_1_SIGMAS[5:])


def _worker(rank: int, size: int, port: int, case: str, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(size),
                      RANK=str(rank), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    from kinomlx_b200 import dist
    from kinomlx_b200.sequence_parallel import SequenceParallel

    dist.init("nccl", timeout_s=120)
    device = torch.device("cuda", rank)
    if case == "cfg":
        from kinomlx_b200.flux2 import sampling
        from kinomlx_b200.flux2.transformer import Flux2Transformer
        from kinomlx_b200.multi_gpu import CfgSplit, cfg_split_step
        from kinomlx_b200.synthetic import normal

        cfg = CfgSplit()
        v, w, noise, text, ids = _flux_case()
        negative = normal(tuple(text.shape), seed=45)
        model = Flux2Transformer(w, v, device, sp=cfg.sp)
        prepared = model.prepare(text if cfg.branch == 0 else negative, ids)
        i0, i1 = cfg.sp.shard(noise.shape[1])
        current = noise[:, i0:i1].to(device).clone()
        sig = sampling.linear_sigmas(3)
        for i in range(3):
            cfg_split_step(model, prepared, current, sig, i, 4.0, cfg)
        out = cfg.sp.all_gather_tokens(current)
    elif case in ("vae", "vae_root"):
        from kinomlx_b200.multi_gpu import decode_tiles_distributed

        dec, latent = _vae_case(device)
        # vae_root: the video assembled on rank 1 only (NCCL reduce); rank 0 returns None
        out = decode_tiles_distributed(dec, latent, tile=4, overlap=1,
                                       dst=1 if case == "vae_root" else None)
    else:
        sp = SequenceParallel(peer=case.endswith("_peer"))
        out = _run(case.removesuffix("_peer"), device, sp)
        torch.cuda.synchronize()
        sp.close()
    torch.cuda.synchronize()
    import torch.distributed as tdist

    tdist.destroy_process_group()
    queue.put((rank, None if out is None else out.float().cpu().numpy().tolist()))


@pytest.mark.parametrize("case", ["flux", "ltx", "flux_peer", "ltx_peer", "cfg", "vae", "vae_root"])
def test_two_gpus_match_one_gpu(cuda_device, case):
    """flux/ltx: Ulysses over 2 ranks through NCCL all-to-alls; *_peer: the same through the
    peer transport (projection epilogues and attention store into the other GPU's buffers over
    NVLink, device barriers); cfg: conditional and unconditional branch on different GPUs with
    the velocity exchange; vae: tiles split over 2 ranks, canvases all-reduced; vae_root: the
    canvases reduced onto rank 1 only."""
    size, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, size, port, case, queue)) for r in range(size)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=600) for _ in range(size))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    expect = _run(case.removesuffix("_peer").removesuffix("_root"), cuda_device).float().cpu()
    for r in range(size):
        if case == "vae_root" and r == 0:
            assert results[r] is None
            continue
        got = torch.tensor(results[r])
        cos = float(torch.nn.functional.cosine_similarity(got.flatten(), expect.flatten(), dim=0))
        max_rel = float((got - expect).abs().max() / expect.abs().max())
        assert cos >= 0.9999 and max_rel <= 1e-2, (case, r, cos, max_rel)
