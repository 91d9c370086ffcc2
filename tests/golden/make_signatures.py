"""Record the call signatures of the reference's pytorch_impl functions.

Run in a container that has the reference checkout (tingxi-li/DSLPerfGap) at
REF (default /root/reference); writes tests/golden/reference_signatures.json:
{"<kernel>": {"<function>": "<inspect.signature string>"}} for every function
the CUDA backend's ViperBench/<kernel>/cuda_impl.py stubs must match.

    python tests/golden/make_signatures.py [REF]
"""
import importlib.util
import inspect
import json
import sys
from pathlib import Path

FUNCTIONS = {
    "layer_norm": ["layer_norm"], "rms_norm": ["rms_norm"], "softmax": ["softmax"],
    "log_softmax": ["log_softmax"], "logsumexp": ["logsumexp"],
    "cross_entropy": ["cross_entropy_fwd", "cross_entropy_bwd"], "mean_reduction": ["mean_reduction"],
    "max_reduction": ["max_reduction"], "argmax": ["argmax"], "linear_activation": ["kernel_ff"],
}


def main(ref: str = "/root/reference") -> None:
    viper = Path(ref) / "ViperBench"
    out = {}
    for kernel, fns in FUNCTIONS.items():
        path = viper / kernel / "pytorch_impl.py"
        spec = importlib.util.spec_from_file_location(f"ref_{kernel}_pytorch_impl", str(path))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        out[kernel] = {fn: str(inspect.signature(getattr(mod, fn))) for fn in fns}
    dst = Path(__file__).resolve().parent / "reference_signatures.json"
    dst.write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print(f"wrote {dst}")


if __name__ == "__main__":
    main(*sys.argv[1:])
