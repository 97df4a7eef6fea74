"""Writes tests/golden/reference_kats.json: the known-answer cases of the
reference's own unit tests for the sampling path, transcribed by hand.

Sources (xUnit, Neuraval.Tests/):
  TokenSamplerTests.cs:10-93, LogitsProcessorTests.cs:9-156 (calls at :14-155),
  GenerationOptionsTests.cs:27-71.
Each case records the file:line it comes from and a literal snippet of that
line. The script checks that every snippet appears on the cited line of the
reference tree (its root in NEURAVAL_REFERENCE) before writing the fixture, so
the transcription is pinned to the source:
  NEURAVAL_REFERENCE=<reference root> python tests/golden/make_reference_kats.py
The C# tests draw with `new Random(seed)`; the cases here only use draws that
the reference pins for every seed (greedy, top-k 1), so any u gives the answer.
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "reference_kats.json")
INT_MAX = 2**31 - 1
TS = "Neuraval.Tests/TokenSamplerTests.cs"
LP = "Neuraval.Tests/LogitsProcessorTests.cs"
GO = "Neuraval.Tests/GenerationOptionsTests.cs"

# GenerationOptions.CreateGreedy(maxNew, stop) = Create(true, 1, 1, int.MaxValue, 1, ...)
GREEDY = dict(greedy=True, temperature=1.0, top_p=1.0, top_k=INT_MAX, repetition_penalty=1.0)

SAMPLER = [
    dict(name="greedy_returns_argmax", src=f"{TS}:13", snippet="new float[] { 1f, 5f, 2f, 4f }",
         logits=[1, 5, 2, 4], history=[], params=GREEDY, uniforms=[0.0, 0.5, 0.99], expect=1),
    dict(name="topk1_returns_highest", src=f"{TS}:24", snippet="new float[] { 1f, 2f, 9f, 3f }",
         logits=[1, 2, 9, 3], history=[],
         params=dict(greedy=False, temperature=0.7, top_p=1.0, top_k=1, repetition_penalty=1.0),
         uniforms=[i / 20 for i in range(20)], expect=2),
    dict(name="repetition_penalty_demotes_sampled", src=f"{TS}:37",
         snippet="new float[] { 5f, 4f, 0f, 0f }", logits=[5, 4, 0, 0], history=[0],
         params=dict(greedy=False, temperature=1.0, top_p=1.0, top_k=1, repetition_penalty=10.0),
         uniforms=[0.0, 0.5, 0.99], expect=1),
    dict(name="greedy_applies_repetition_penalty", src=f"{TS}:51",
         snippet="GenerationOptions.Create(true, 1f, 1f, int.MaxValue, 10f",
         logits=[5, 4, 0, 0], history=[0],
         params=dict(greedy=True, temperature=1.0, top_p=1.0, top_k=INT_MAX,
                     repetition_penalty=10.0), uniforms=[0.3], expect=1),
    dict(name="greedy_penalty_one_keeps_argmax", src=f"{TS}:63",
         snippet="GenerationOptions.Create(true, 1f, 1f, int.MaxValue, 1f",
         logits=[5, 4, 0, 0], history=[0],
         params=dict(greedy=True, temperature=1.0, top_p=1.0, top_k=INT_MAX,
                     repetition_penalty=1.0), uniforms=[0.3], expect=0),
]

PROCESSOR = [
    dict(op="repetition_penalty", src=f"{LP}:14", snippet="Array.Empty<int>(), 1.5f",
         logits=[1, 2, 3], history=[], arg=1.5, expect=[1, 2, 3]),
    dict(op="repetition_penalty", src=f"{LP}:24", snippet="new[] { 0, 1 }, 1f",
         logits=[1, 2, 3], history=[0, 1], arg=1.0, expect=[1, 2, 3]),
    dict(op="repetition_penalty", src=f"{LP}:34", snippet="new[] { 0 }, 2f",
         logits=[4, 2], history=[0], arg=2.0, expect=[2, 2]),
    dict(op="repetition_penalty", src=f"{LP}:45", snippet="new[] { 0 }, 2f",
         logits=[-4], history=[0], arg=2.0, expect=[-8]),
    dict(op="repetition_penalty", src=f"{LP}:55", snippet="new[] { 0, 0, 0 }, 2f",
         logits=[8], history=[0, 0, 0], arg=2.0, expect=[4]),
    dict(op="repetition_penalty", src=f"{LP}:64", snippet="new[] { 0 }, 0f",
         logits=[1], history=[0], arg=0.0, expect="invalid"),
    dict(op="temperature", src=f"{LP}:72", snippet="ApplyTemperature(logits, 1f)",
         logits=[1, -2], arg=1.0, expect=[1, -2]),
    dict(op="temperature", src=f"{LP}:82", snippet="ApplyTemperature(logits, 2f)",
         logits=[4, -2], arg=2.0, expect=[2, -1]),
    dict(op="temperature", src=f"{LP}:91", snippet="new float[] { 1f }, 0f",
         logits=[1], arg=0.0, expect="invalid"),
    dict(op="filter_top_k", src=f"{LP}:99", snippet="FilterTopK(logits, 2)",
         logits=[1, 5, 3, 2, 4], arg=2, expect=["-inf", 5, "-inf", "-inf", 4]),
    dict(op="filter_top_k", src=f"{LP}:113", snippet="FilterTopK(logits, 10)",
         logits=[1, 2, 3], arg=10, expect=[1, 2, 3]),
    dict(op="filter_top_k", src=f"{LP}:122", snippet="new float[] { 1f }, 0",
         logits=[1], arg=0, expect="invalid"),
    # FilterTopP asserts: entries 2,3 are 0, entries 0,1 positive, sum 1 to 5 digits
    dict(op="filter_top_p", src=f"{LP}:130", snippet="FilterTopP(probabilities, 0.8f)",
         logits=[0.5, 0.3, 0.1, 0.1], arg=0.8, expect="nucleus_2_renormalised"),
    dict(op="filter_top_p", src=f"{LP}:146", snippet="FilterTopP(probabilities, 1f)",
         logits=[0.5, 0.3, 0.2], arg=1.0, expect=[0.5, 0.3, 0.2]),
    dict(op="filter_top_p", src=f"{LP}:155", snippet="new float[] { 1f }, 0f",
         logits=[1], arg=0.0, expect="invalid"),
]

# GenerationOptions.Create validation (the reference throws ArgumentOutOfRange)
OPTIONS = [
    dict(src=f"{GO}:28", snippet="[InlineData(0f)]", field="temperature", value=0.0),
    dict(src=f"{GO}:29", snippet="[InlineData(-1f)]", field="temperature", value=-1.0),
    dict(src=f"{GO}:37", snippet="[InlineData(0f)]", field="top_p", value=0.0),
    dict(src=f"{GO}:38", snippet="[InlineData(-0.1f)]", field="top_p", value=-0.1),
    dict(src=f"{GO}:39", snippet="[InlineData(1.1f)]", field="top_p", value=1.1),
    dict(src=f"{GO}:47", snippet="[InlineData(0)]", field="top_k", value=0),
    dict(src=f"{GO}:48", snippet="[InlineData(-5)]", field="top_k", value=-5),
    dict(src=f"{GO}:56", snippet="[InlineData(0f)]", field="repetition_penalty", value=0.0),
    dict(src=f"{GO}:57", snippet="[InlineData(-1f)]", field="repetition_penalty", value=-1.0),
]
# the base options of those theories: Create(false, 0.7f, 0.9f, 40, 1f, 10, ...)
OPTIONS_BASE = dict(greedy=False, temperature=0.7, top_p=0.9, top_k=40, repetition_penalty=1.0)


def verify(root: str) -> int:
    bad = 0
    for case in SAMPLER + PROCESSOR + OPTIONS:
        path, line = case["src"].rsplit(":", 1)
        with open(os.path.join(root, path), encoding="utf-8") as fh:
            text = fh.read().splitlines()[int(line) - 1]
        if case["snippet"] not in text:
            print(f"MISMATCH {case['src']}: {case['snippet']!r} not in {text.strip()!r}")
            bad += 1
    return bad


def main() -> int:
    root = os.environ.get("NEURAVAL_REFERENCE")
    if not root or not os.path.isdir(root):
        print("set NEURAVAL_REFERENCE to the reference tree's root: every citation is "
              "checked against it before the fixture is written", file=sys.stderr)
        return 1
    bad = verify(root)
    if bad:
        return 1
    print(f"verified {len(SAMPLER) + len(PROCESSOR) + len(OPTIONS)} citations against {root}")
    with open(OUT, "w") as fh:
        json.dump(dict(sampler=SAMPLER, processor=PROCESSOR, options=OPTIONS,
                       options_base=OPTIONS_BASE), fh, indent=1)
    print(f"wrote {OUT}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
