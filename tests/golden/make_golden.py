"""Generates tests/golden/prototype_golden.npz from the reference's own
PyTorch prototype (src/diffusion.py:6-10 timestep_embedding, src/vae.py:7-15
ResBlock with SiLU, and the decoder's / encoder's stages src/vae.py:44-45
Decoder._up -- ResBlock, nearest x2 upsample, 3x3 conv, SiLU -- and
src/vae.py:27-28 Encoder._down -- ResBlock, stride-2 3x3 conv, SiLU -- with
their autograd gradients for an upstream gradient g; and the time
conditioning of src/diffusion.py:38,49 -- DiT.time_mlp, Linear -> SiLU ->
Linear, over timestep_embedding -- with its weight gradients).  Run where
the reference checkout is available:

    python tests/golden/make_golden.py /path/to/YumeLayers

The committed .npz is what the tests read; nothing at test time imports the
reference.
"""
import sys
from pathlib import Path

import numpy as np
import torch


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    from config import Config  # noqa: E402  (reference prototype)
    from diffusion import DiT, timestep_embedding  # noqa: E402
    from vae import Decoder, Encoder, ResBlock  # noqa: E402

    torch.manual_seed(0)
    rng = np.random.default_rng(0)
    t = rng.uniform(0, 1000, 7).astype(np.float32)
    temb = timestep_embedding(torch.tensor(t), 128).numpy()

    block = ResBlock(8)
    x = rng.standard_normal((2, 8, 6, 7)).astype(np.float32)
    with torch.no_grad():
        y = block(torch.tensor(x)).numpy()
    conv1, conv2 = block.net[0], block.net[2]
    arrays = dict(
        temb_t=t, temb_out=temb.astype(np.float32), rb_x=x,
        rb_w1=conv1.weight.detach().numpy(), rb_b1=conv1.bias.detach().numpy(),
        rb_w2=conv2.weight.detach().numpy(), rb_b2=conv2.bias.detach().numpy(),
        rb_y=y.astype(np.float32))
    # one decoder stage (8 -> 4 channels, 5x6 -> 10x12) and one encoder stage
    # (8 -> 16 channels, 7x9 -> 4x5), forward and backward
    stages = (("up", Decoder(base=4)._up(8, 4), (2, 8, 5, 6)),
              ("down", Encoder(base=4)._down(8, 16), (2, 8, 7, 9)))
    for name, stage, shape in stages:
        xs = torch.tensor(rng.standard_normal(shape).astype(np.float32), requires_grad=True)
        ys = stage(xs)
        g = torch.tensor(rng.standard_normal(tuple(ys.shape)).astype(np.float32))
        (ys * g).sum().backward()
        rb = stage[0].net
        conv = stage[2] if name == "up" else stage[1]
        for key, mod in (("rb_w1", rb[0]), ("rb_w2", rb[2]), ("w", conv)):
            arrays[f"{name}_{key}"] = mod.weight.detach().numpy()
            arrays[f"{name}_{key.replace('w', 'b')}"] = mod.bias.detach().numpy()
            arrays[f"{name}_d{key}"] = mod.weight.grad.numpy()
            arrays[f"{name}_d{key.replace('w', 'b')}"] = mod.bias.grad.numpy()
        arrays[f"{name}_x"] = xs.detach().numpy()
        arrays[f"{name}_y"] = ys.detach().numpy()
        arrays[f"{name}_g"] = g.numpy()
        arrays[f"{name}_dx"] = xs.grad.numpy()
    # the DiT's time conditioning at its default width (128)
    cfg = Config()
    mlp = DiT(cfg).time_mlp
    tt = torch.tensor(rng.uniform(0, 200, 5).astype(np.float32))
    emb = timestep_embedding(tt, cfg.dif_dim)
    ym = mlp(emb)
    gm = torch.tensor(rng.standard_normal(tuple(ym.shape)).astype(np.float32))
    (ym * gm).sum().backward()
    for key, mod in (("w1", mlp[0]), ("w2", mlp[2])):
        arrays[f"tmlp_{key}"] = mod.weight.detach().numpy()
        arrays[f"tmlp_{key.replace('w', 'b')}"] = mod.bias.detach().numpy()
        arrays[f"tmlp_d{key}"] = mod.weight.grad.numpy()
        arrays[f"tmlp_d{key.replace('w', 'b')}"] = mod.bias.grad.numpy()
    arrays["tmlp_t"] = tt.numpy()
    arrays["tmlp_y"] = ym.detach().numpy()
    arrays["tmlp_g"] = gm.numpy()
    out = Path(__file__).resolve().parent / "prototype_golden.npz"
    np.savez_compressed(out, **arrays)
    print("wrote", out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/YumeLayers")
    main(sys.argv[1])
