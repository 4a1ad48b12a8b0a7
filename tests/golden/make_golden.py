"""Generates tests/golden/prototype_golden.npz from the reference's own
PyTorch prototype (src/diffusion.py:6-10 timestep_embedding, src/vae.py:7-15
ResBlock with SiLU).  Run where the reference checkout is available:

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
    from diffusion import timestep_embedding  # noqa: E402  (reference prototype)
    from vae import ResBlock  # noqa: E402

    torch.manual_seed(0)
    rng = np.random.default_rng(0)
    t = rng.uniform(0, 1000, 7).astype(np.float32)
    temb = timestep_embedding(torch.tensor(t), 128).numpy()

    block = ResBlock(8)
    x = rng.standard_normal((2, 8, 6, 7)).astype(np.float32)
    with torch.no_grad():
        y = block(torch.tensor(x)).numpy()
    conv1, conv2 = block.net[0], block.net[2]
    out = Path(__file__).resolve().parent / "prototype_golden.npz"
    np.savez_compressed(
        out, temb_t=t, temb_out=temb.astype(np.float32), rb_x=x,
        rb_w1=conv1.weight.detach().numpy(), rb_b1=conv1.bias.detach().numpy(),
        rb_w2=conv2.weight.detach().numpy(), rb_b2=conv2.bias.detach().numpy(),
        rb_y=y.astype(np.float32))
    print("wrote", out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/YumeLayers")
    main(sys.argv[1])
