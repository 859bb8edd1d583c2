"""The cgo shims (stream-pt_b200/go/*.go: the MoE block, the Q4_0 products and
the Q8_0 head) against the reference's Go API and the C ABI, without a Go
toolchain (none is installed here).

Every identifier the shim takes from package forward, ggufindex or ggufmap
must exist in the reference (tests/golden/go_api.json, written from the
reference sources by tests/golden/make_go_api.py), forwardMoEBatch must keep
the reference's parameter list, and every C function and struct field it
uses must be declared in include/spt_moe.h.
"""
import json
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GO_DIR = os.path.join(ROOT, "stream-pt_b200", "go")
SHIMS = {f: open(os.path.join(GO_DIR, f)).read() for f in sorted(os.listdir(GO_DIR)) if f.endswith(".go")}
SHIM = SHIMS["moe_cuda.go"]
API = json.load(open(os.path.join(ROOT, "tests", "golden", "go_api.json")))
HEADER = open(os.path.join(ROOT, "include", "spt_moe.h")).read()
# every shim file, comments out (they form one package)
CODE = "\n".join(re.sub(r"//[^\n]*", "", src) for src in SHIMS.values())
Q40 = re.sub(r"//[^\n]*", "", SHIMS["q40_cuda.go"])
Q80 = re.sub(r"//[^\n]*", "", SHIMS["q80_cuda.go"])


def test_imports_name_the_reference_packages():
    for src in SHIMS.values():
        code = re.sub(r"//[^\n]*", "", src)
        imports = dict((alias or path.split("/")[-1], path) for alias, path in
                       re.findall(r'^\s*(\w+)?\s*"([^"]+)"$', code.split("import (", 1)[1].split(")", 1)[0], re.M))
        assert imports["ggufindex"] == API["module"] + "/ggufindex"
        assert imports[API["packages"]["ggufmap"]] == API["module"] + "/ggufmap"
        assert src.startswith("//go:build goexperiment.simd && sptcuda")


def test_reader_methods_exist():
    used = set(re.findall(r"\breader\.(\w+)\(", CODE))
    assert used and used <= set(API["reader_methods"]), used - set(API["reader_methods"])
    assert "WithFile" not in used
    # WithTensor's callback is func(data []byte) error
    assert API["with_tensor"] == "t ggufindex.Tensor, fn func(data []byte) error"
    assert re.search(r"reader\.WithTensor\(\w+\[0\], func\(data \[\]byte\) error \{", CODE)


def test_fields_exist():
    checks = [(r"\blw\.(\w+)", "layer_weights_fields"), (r"\bcfg\.(\w+)", "config_fields"),
              (r"\bt\.(\w+)", "tensor_fields"), (r"\bts\[\d+\]\.(\w+)", "tensor_fields"),
              (r"\btensor\.(\w+)", "tensor_fields"), (r"\boptions\.(\w+)", "q40_options_fields"),
              (r"\.Range\.(\w+)", "range_fields")]
    for pat, key in checks:
        used = set(re.findall(pat, CODE))
        assert used <= set(API[key]), (key, used - set(API[key]))
    for pkg, key in (("ggufindex", "ggufindex_exported"), (API["packages"]["ggufmap"], "ggufmap_exported")):
        used = set(re.findall(r"\b%s\.(\w+)" % pkg, CODE))
        assert used <= set(API[key]), (pkg, used - set(API[key]))
    for typ in ("Config", "LayerWeights", "Q40Options", "moeBatchScratch"):
        assert typ in API["forward_types"]


def test_forward_moe_batch_signature_unchanged():
    sig = re.search(r"func forwardMoEBatch\((.*?)\) error \{", CODE, re.S).group(1)
    assert " ".join(sig.split()) == API["forward_moe_batch_params"]


def test_c_symbols_and_fields_are_declared():
    funcs = set(re.findall(r"\b(spt_\w+)\s*\(", HEADER))
    consts = set(re.findall(r"#define (SPT_\w+)", HEADER)) | set(re.findall(r"\b(SPT_(?:OK|ERR_\w+))\b", HEADER))
    types = set(re.findall(r"typedef struct (spt_\w+)", HEADER))
    used_funcs = set(re.findall(r"\bC\.(spt_[a-z_]+)\(", CODE)) - types
    assert used_funcs and used_funcs <= funcs, used_funcs - funcs
    used_consts = set(re.findall(r"\bC\.(SPT_\w+)", CODE))
    assert used_consts <= consts, used_consts - consts
    for typ in set(re.findall(r"(?<!\*)\bC\.(spt_\w+)\{", CODE)):  # composite literals (not map[..]*C.x{})
        body = re.search(r"typedef struct %s \{(.*?)\}" % typ, HEADER, re.S).group(1)
        fields = set(re.findall(r"\b([a-z_]\w*)\s*[,;\[]", body))
        for m in re.finditer(r"C\.%s\{" % typ, CODE):
            depth, i = 1, m.end()
            while depth:  # the literal's own braces
                depth += {"{": 1, "}": -1}.get(CODE[i], 0)
                i += 1
            block = CODE[m.end():i - 1]
            named = set(re.findall(r"\b([a-z_]\w*):", block))
            assert named <= fields, (typ, named - fields)


def test_q40_signatures_unchanged():
    """MulQ40Into / MulQ40BatchInto keep the reference's parameter lists
    (forward/q40.go:35-101); the helpers the shim keeps from q40.go exist."""
    one = re.search(r"func MulQ40Into\((.*?)\) error \{", Q40, re.S).group(1)
    many = re.search(r"func MulQ40BatchInto\((.*?)\) error \{", Q40, re.S).group(1)
    assert " ".join(one.split()) == API["mul_q40_params"]
    assert " ".join(many.split()) == API["mul_q40_batch_params"]
    assert API["q40_shape_results"] == "input, output, rowBytes int, err error"
    assert re.search(r"input, output, rowBytes, err := q40Shape\(tensor\)", Q40)
    for fn in ("q40Shape", "float32Overlap"):
        assert fn in API["forward_funcs"]
    assert "DefaultQ40WindowBytes" in API["forward_consts"]
    # the shim defines only the two replaced exported functions and its helpers
    defined = set(re.findall(r"^func (\w+)\(", Q40, re.M))
    assert defined == {"q40Matrix", "MulQ40Into", "MulQ40BatchInto"}


def test_q40_error_texts_follow_the_reference():
    for text in ("nil context", "nil GGUF reader", "invalid or oversized batch: %d",
                 "%q: expected %d input and %d output elements, got %d and %d",
                 "input and output must not overlap", "window of %d bytes cannot accommodate a %d-byte row"):
        assert '"%s"' % text in Q40, text


def test_q80_signatures_unchanged():
    """MulQ80Argmax / MulQ80Into keep the reference's parameter and result
    lists (forward/q80.go:20-148); the helpers the shim keeps from q80.go
    exist."""
    argmax = re.search(r"func MulQ80Argmax\((.*?)\) \((.*?)\) \{", Q80, re.S)
    into = re.search(r"func MulQ80Into\((.*?)\) error \{", Q80, re.S).group(1)
    assert " ".join(argmax.group(1).split()) == API["mul_q80_argmax_params"]
    assert " ".join(argmax.group(2).split()) == API["mul_q80_argmax_results"]
    assert " ".join(into.split()) == API["mul_q80_into_params"]
    assert API["q80_shape_results"] == "input, output, rowBytes int, err error"
    assert len(re.findall(r"input, output, rowBytes, err := q80Shape\(tensor\)", Q80)) == 2
    assert "q80Shape" in API["forward_funcs"] and "DefaultQ40WindowBytes" in API["forward_consts"]
    defined = set(re.findall(r"^func (\w+)\(", Q80, re.M))
    assert defined == {"q80Matrix", "q80Window", "mulQ80", "MulQ80Argmax", "MulQ80Into"}
    # no helper of the same name elsewhere in the shims (one package)
    others = "\n".join(re.sub(r"//[^\n]*", "", v) for k, v in SHIMS.items() if k != "q80_cuda.go")
    for fn in defined:
        assert not re.search(r"^func %s\(" % fn, others, re.M), fn


def test_q80_error_texts_follow_the_reference():
    for text in ("nil context", "nil reader", "nil context or reader",
                 "%q: expected %d input elements, got %d",
                 "%q: expected input/output lengths %d/%d, got %d/%d",
                 "window of %d bytes cannot accommodate a %d-byte row"):
        assert '"%s"' % text in Q80, text


def test_library_calls_hold_the_call_lock():
    """Every call into the shared context (uploads and products) and every
    read of its error text runs between sptCallM.Lock() and its Unlock: the
    calls share one stream, its device buffers and its last-error text.  A
    "defer sptCallM.Unlock()" holds the lock to the end of its block."""
    exempt = {"spt_context_create", "spt_last_error"}  # under sync.Once / inside sptError
    for name, src in SHIMS.items():
        locked, defer_indent = False, None
        for n, line in enumerate(src.splitlines(), 1):
            code = line.split("//")[0]
            indent = len(line) - len(line.lstrip("\t"))
            if defer_indent is not None and code.strip() and indent < defer_indent:
                locked, defer_indent = False, None
            if "sptCallM.Lock()" in code:
                locked = True
            if "defer sptCallM.Unlock()" in code:
                defer_indent = indent
            elif "sptCallM.Unlock()" in code:
                locked = False
            calls = set(re.findall(r"\bC\.(spt_[a-z_0-9]+)\(", code)) - exempt
            if calls or (re.search(r"\bsptError\(", code) and not code.startswith("func ")):
                assert locked, f"{name}:{n}: {line.strip()}"

