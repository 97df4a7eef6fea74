"""Writes the reference's known-answer cases (tests/golden/reference_kats.json,
each with its source line) as C++ initialisers for host_mirror_tests.cpp."""
import json
import math
import sys


def fl(x):
    if isinstance(x, str):
        return {"-inf": "-INFINITY", "inf": "INFINITY"}[x]
    if math.isinf(x):
        return "INFINITY" if x > 0 else "-INFINITY"
    return repr(float(x)) + "f"


def vec_f(xs):
    return "{" + ", ".join(fl(x) for x in xs) + "}"


def vec_i(xs):
    return "{" + ", ".join(str(int(x)) for x in xs) + "}"


def main(src, dst):
    k = json.load(open(src))
    out = ["// generated from tests/golden/reference_kats.json by tests/cpp/gen_kats.py"]
    out.append("static const SamplerKat kSamplerKats[] = {")
    for c in k["sampler"]:
        p = c["params"]
        out.append("  {%r, %s, %s, %s, %s, %s, %d, %s, %s, %d}," % (
            c["src"], vec_f(c["logits"]), vec_i(c["history"]), "true" if p["greedy"] else "false",
            fl(p["temperature"]), fl(p["top_p"]), min(int(p["top_k"]), 2**31 - 1),
            fl(p["repetition_penalty"]), vec_f(c["uniforms"]), int(c["expect"])))
    out.append("};")
    out.append("static const ProcessorKat kProcessorKats[] = {")
    for c in k["processor"]:
        exp = c["expect"]
        kind = "kInvalid" if exp == "invalid" else ("kNucleus2" if exp == "nucleus_2_renormalised"
                                                     else "kValues")
        vals = vec_f(exp) if kind == "kValues" else "{}"
        out.append("  {%r, %r, %s, %s, %s, %s, %s}," % (
            c["src"], c["op"], vec_f(c["logits"]), vec_i(c.get("history") or []), fl(c["arg"]),
            kind, vals))
    out.append("};")
    b = k["options_base"]
    out.append("static const OptionsBase kOptionsBase = {%s, %s, %s, %d, %s};" % (
        "true" if b["greedy"] else "false", fl(b["temperature"]), fl(b["top_p"]), int(b["top_k"]),
        fl(b["repetition_penalty"])))
    out.append("static const OptionsKat kOptionsKats[] = {")
    for c in k["options"]:
        out.append("  {%r, %r, %s}," % (c["src"], c["field"], fl(c["value"])))
    out.append("};")
    text = "\n".join(out).replace("'", '"') + "\n"
    open(dst, "w").write(text)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
