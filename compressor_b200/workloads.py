"""Seeded synthetic client updates with the shapes of the benchmark models.

The reference's replay datasets are not available, so these generators stand
in for them (same tensor names, shapes and count as the reference's
ResNet-18 / ResNet-50 state-dict manifests, GPT-2-medium shapes from the
architecture):

* ``resnet18`` / ``resnet50``: round 0 per tensor N(0, (1e-3/sqrt(fan_in))^2);
  round t: d_t = rho * d_{t-1} + N(0, same sigma^2), rho = 0.9.
* ``microbench``: one 512x512x3x3 tensor, sigma = 1e-4, rho = 0.9.
* ``gpt2-medium``: Student-t (nu = 3) scaled by 1e-4, rho = 0.8
  (``gpt2-medium-slice``: the same for the embedding tables, the first block
  and the final layer norm only).
* multi-client federations add a shared N(0, (1e-3)^2) component per round.

Draws are float32 from numpy PCG64 with fixed seeds; the same host bytes feed
the GPU codec and the CPU checker.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, List, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def manifest(model: str) -> List[Tuple[str, Tuple[int, ...]]]:
    if model in ("resnet18", "resnet50"):
        out = []
        with open(os.path.join(HERE, "manifests", f"{model}.tsv")) as f:
            for line in f:
                name, shape = line.rstrip("\n").split("\t")
                out.append((name, tuple(int(x) for x in shape.split("x"))))
        return out
    if model == "microbench":
        return [("layer4.0.conv2.weight", (512, 512, 3, 3))]
    if model in ("gpt2-medium", "gpt2-medium-slice"):
        # the slice: both full-size embedding tables, the first block and the
        # final layer norm (the parity tests' subset)
        d, vocab, npos, L = 1024, 50257, 1024, 24 if model == "gpt2-medium" else 1
        out = [("transformer.wte.weight", (vocab, d)), ("transformer.wpe.weight", (npos, d))]
        for i in range(L):
            p = f"transformer.h.{i}."
            out += [
                (p + "ln_1.weight", (d,)), (p + "ln_1.bias", (d,)),
                (p + "attn.c_attn.weight", (d, 3 * d)), (p + "attn.c_attn.bias", (3 * d,)),
                (p + "attn.c_proj.weight", (d, d)), (p + "attn.c_proj.bias", (d,)),
                (p + "ln_2.weight", (d,)), (p + "ln_2.bias", (d,)),
                (p + "mlp.c_fc.weight", (d, 4 * d)), (p + "mlp.c_fc.bias", (4 * d,)),
                (p + "mlp.c_proj.weight", (4 * d, d)), (p + "mlp.c_proj.bias", (d,)),
            ]
        out += [("transformer.ln_f.weight", (d,)), ("transformer.ln_f.bias", (d,))]
        return out
    raise KeyError(model)


def fan_in(shape: Tuple[int, ...]) -> int:
    return int(np.prod(shape[1:])) if len(shape) >= 2 else int(shape[0])


@dataclass
class Layout:
    """All tensors of one update packed back to back in one float32 buffer
    (offsets aligned to 64 elements = 256 bytes)."""
    names: List[str]
    shapes: List[Tuple[int, ...]]
    offsets: List[int]
    total: int

    @staticmethod
    def of(model: str) -> "Layout":
        names, shapes, offs = [], [], []
        off = 0
        for name, shape in manifest(model):
            names.append(name)
            shapes.append(shape)
            offs.append(off)
            off += (int(np.prod(shape)) + 63) // 64 * 64
        return Layout(names, shapes, offs, off)

    def views(self, flat: np.ndarray) -> List[np.ndarray]:
        return [flat[o:o + int(np.prod(s))].reshape(s) for o, s in zip(self.offsets, self.shapes)]

    @property
    def numel(self) -> int:
        return int(sum(int(np.prod(s)) for s in self.shapes))


class UpdateStream:
    """Yields one flat float32 update per round for one client."""

    def __init__(self, model: str, seed: int, rho: float = None, dist: str = None,
                 common_std: float = 0.0, common_seed: int = 12345):
        self.model = model
        self.layout = Layout.of(model)
        self.rng = np.random.Generator(np.random.PCG64(seed))
        self.common = np.random.Generator(np.random.PCG64(common_seed)) if common_std > 0 else None
        self.common_std = common_std
        if model.startswith("gpt2-medium"):
            self.rho = 0.8 if rho is None else rho
            self.dist = dist or "student_t3"
        else:
            self.rho = 0.9 if rho is None else rho
            self.dist = dist or "normal"
        self.sigma = np.zeros(self.layout.total, np.float32)
        self.mask = np.zeros(self.layout.total, bool)
        for o, s in zip(self.layout.offsets, self.layout.shapes):
            n = int(np.prod(s))
            self.mask[o:o + n] = True
            if model == "microbench" or self.dist == "student_t3":
                self.sigma[o:o + n] = 1e-4
            else:
                self.sigma[o:o + n] = 1e-3 / np.sqrt(fan_in(s))
        self.state = None

    def _noise(self) -> np.ndarray:
        if self.dist == "student_t3":
            return (self.rng.standard_t(3, self.layout.total).astype(np.float32) * self.sigma)
        return self.rng.standard_normal(self.layout.total, dtype=np.float32) * self.sigma

    def next(self) -> np.ndarray:
        if self.state is None:
            self.state = self._noise()
        else:
            self.state = np.float32(self.rho) * self.state + self._noise()
        out = self.state
        if self.common is not None:
            out = out + self.common.standard_normal(self.layout.total, dtype=np.float32) * np.float32(self.common_std)
        flat = np.where(self.mask, out, np.float32(0.0)).astype(np.float32)
        return flat


def rounds(model: str, n_rounds: int, seed: int = 0, **kw) -> List[np.ndarray]:
    st = UpdateStream(model, seed, **kw)
    return [st.next() for _ in range(n_rounds)]


def algorithmic_bytes(model: str, codec: str = "q8") -> Dict[str, float]:
    """Bytes one closed-loop round must move through HBM (encoder + decoder),
    assuming every kernel of a momentum layer is predicted:
      momentum element: encoder reads cur/prev/mem (12 B), writes mem and the
      history copy (8 B) and its code q; decoder reads q, prev and mem (8 B +
      q) and writes mem, output and history (12 B) => 40 + 2q B;
      conv kernel: bitmap + dominant-sign bit, written and read (4 bits);
      direct element: encoder reads 4 B, writes history 4 B and payload q;
      decoder reads q and writes output and history 8 B => 16 + 2q B."""
    q = {"q8": 1.0, "int4": 0.5, "raw": 4.0}[codec]
    mom_elems = kernels = direct = 0
    for name, shape in manifest(model):
        n = int(np.prod(shape))
        if len(shape) == 4 and "weight" in name and n > 1024:
            mom_elems += n
            kernels += shape[0] * shape[1]
        else:
            direct += n
    total = mom_elems * (40 + 2 * q) + kernels * 4 / 8 + direct * (16 + 2 * q)
    return {"momentum_elements": mom_elems, "kernels": kernels, "direct_elements": direct,
            "bytes_per_round": total}
