"""Regenerates the ResNet-18 / ResNet-50 state-dict shape manifests.

Reads the layer name / shape table that the reference published with its
CUDA experiments (logs/cuda_v4_guarded_all_cuda/layer_backend_diff.csv under
the reference checkout given as the first argument) and writes one
``name<TAB>d0xd1x...`` line per tensor, in state-dict order.
"""
import csv
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    src = os.path.join(ref_root, "logs", "cuda_v4_guarded_all_cuda", "layer_backend_diff.csv")
    rows = {}
    with open(src) as f:
        for r in csv.DictReader(f):
            rows.setdefault(r["model"], []).append((r["layer_name"], r["shape"]))
    for model, layers in rows.items():
        with open(os.path.join(HERE, f"{model}.tsv"), "w") as out:
            for name, shape in layers:
                out.write(f"{name}\t{shape}\n")
        print(model, len(layers))


if __name__ == "__main__":
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle.reference_root import reference_root
    main(sys.argv[1] if len(sys.argv) > 1 else reference_root())
