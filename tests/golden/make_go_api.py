"""Writes tests/golden/go_api.json: the identifiers of the Stream-PT Go
sources that the cgo shims (stream-pt_b200/go/*.go) rely on, read
from a checkout of the reference (argv[1], else the STREAM_PT_SOURCE
environment variable).
tests/test_go_shim.py checks the shim against this file, so the check runs
where the reference is absent.

    python tests/golden/make_go_api.py path-to-Stream-PT
"""
import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def read(root, rel):
    with open(os.path.join(root, rel)) as f:
        return f.read()


def struct_fields(src, name):
    m = re.search(r"type %s struct \{(.*?)\n\}" % name, src, re.S)
    fields = []
    for line in m.group(1).splitlines():
        line = line.split("//")[0].strip()
        if not line:
            continue
        names = line.split()[0] if "," not in line.split()[0] else line
        for n in re.findall(r"\b([A-Za-z_]\w*)\b", line.split(" ")[0] if "," not in line else line.split(" ")[0]):
            fields.append(n)
        if "," in line:  # "a, b, c int" forms
            head = re.match(r"([\w\s,]+?)\s+[\[\]\*\w.]+$", line)
            if head:
                fields.extend(x.strip() for x in head.group(1).split(","))
    return sorted(set(f for f in fields if f))


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("STREAM_PT_SOURCE", "")
    if not root:
        sys.exit("usage: make_go_api.py path-to-Stream-PT (or set STREAM_PT_SOURCE)")
    gomod = read(root, "go.mod")
    module = re.search(r"^module\s+(\S+)", gomod, re.M).group(1)
    mm = read(root, "ggufmap/mmap_linux.go")
    idx = read(root, "ggufindex/index.go")
    layer = read(root, "forward/layer.go")
    config = read(root, "forward/config.go")
    batch = read(root, "forward/moe_batch.go")
    q40 = "".join(read(root, os.path.join("forward", f)) for f in os.listdir(os.path.join(root, "forward"))
                  if f.endswith(".go"))
    sig = re.search(r"func forwardMoEBatch\((.*?)\) error \{", batch, re.S).group(1)
    api = {
        "module": module,
        "packages": {"ggufindex": re.search(r"^package (\w+)", idx, re.M).group(1),
                     "ggufmap": re.search(r"^package (\w+)", mm, re.M).group(1)},
        "reader_methods": sorted(set(re.findall(r"^func \(r \*Reader\) ([A-Z]\w*)\(", mm, re.M))),
        "with_tensor": re.search(r"^func \(r \*Reader\) WithTensor\((.*?)\) \(", mm, re.M).group(1),
        "ggufindex_exported": sorted(set(re.findall(r"^(?:type|func) ([A-Z]\w*)", idx, re.M))),
        "ggufmap_exported": sorted(set(re.findall(r"^(?:type|func) ([A-Z]\w*)", mm, re.M))),
        "tensor_fields": struct_fields(idx, "Tensor"),
        "range_fields": struct_fields(idx, "Range"),
        "layer_weights_fields": struct_fields(layer, "LayerWeights"),
        "config_fields": struct_fields(config, "Config"),
        "q40_options_fields": struct_fields(q40, "Q40Options"),
        "forward_types": sorted(set(re.findall(r"^type (\w+)", q40, re.M))),
        "forward_moe_batch_params": " ".join(sig.split()),
        "forward_funcs": sorted(set(re.findall(r"^func ([A-Za-z]\w*)\(", q40, re.M))),
        "forward_consts": sorted(set(re.findall(r"^(?:const |\t)([A-Za-z]\w*)\s*(?:[\w.]+\s*)?=", q40, re.M))),
        "mul_q40_params": " ".join(re.search(r"func MulQ40Into\((.*?)\) error \{", q40, re.S).group(1).split()),
        "mul_q40_batch_params": " ".join(
            re.search(r"func MulQ40BatchInto\((.*?)\) error \{", q40, re.S).group(1).split()),
        "q40_shape_results": " ".join(
            re.search(r"func q40Shape\(tensor ggufindex\.Tensor\) \((.*?)\) \{", q40, re.S).group(1).split()),
        "mul_q80_argmax_params": " ".join(
            re.search(r"func MulQ80Argmax\((.*?)\) \(", q40, re.S).group(1).split()),
        "mul_q80_argmax_results": " ".join(
            re.search(r"func MulQ80Argmax\(.*?\) \((.*?)\) \{", q40, re.S).group(1).split()),
        "mul_q80_into_params": " ".join(re.search(r"func MulQ80Into\((.*?)\) error \{", q40, re.S).group(1).split()),
        "q80_shape_results": " ".join(
            re.search(r"func q80Shape\(tensor ggufindex\.Tensor\) \((.*?)\) \{", q40, re.S).group(1).split()),
    }
    with open(os.path.join(HERE, "go_api.json"), "w") as f:
        json.dump(api, f, indent=1, sort_keys=True)
        f.write("\n")


if __name__ == "__main__":
    main()
