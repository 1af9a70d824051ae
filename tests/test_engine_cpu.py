"""CPU tier: the engine's request rules (include/zcgvs/engine/vector_engine.hpp), compiled into a
small host program (tests/cpp/engine_rules.cpp) and checked against the reference Engine's rules
restated here: option resolution (src/engine/engine.cpp:87-126), lexical term preparation
(:150-172) and the allow mask (:128-146)."""

from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def rules(tmp_path_factory):
    exe = tmp_path_factory.mktemp("engine") / "engine_rules"
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cxx = shutil.which("g++") or shutil.which("c++")
    subprocess.run([cxx, "-std=c++17", "-O1", f"-I{ROOT / 'include'}", f"-I{cuda}/include",
                    str(ROOT / "tests/cpp/engine_rules.cpp"), "-o", str(exe)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines()
    return out


def resolved(lines, name):
    line = next(l for l in lines if l.startswith(name + " "))
    return dict(kv.split("=") for kv in line.split()[1:])


def expect(top_k, candidates, rescore, weight, hybrid, graph, metric):
    return {"top_k": str(top_k), "candidates": str(candidates), "rescore": str(rescore), "weight": f"{weight:.3f}",
            "hybrid": str(hybrid), "graph": str(graph), "metric": str(metric)}


@pytest.mark.parametrize("name,want", [
    ("defaults", expect(10, 100, 0, 0.7, 0, 0, 0)),
    ("small_corpus", expect(10, 50, 0, 0.7, 0, 0, 0)),              # candidates capped at the corpus
    ("topk_over_candidates", expect(200, 200, 0, 0.7, 0, 0, 0)),    # candidates raised to top_k
    ("topk_over_corpus", expect(150, 150, 0, 0.7, 0, 0, 0)),        # both capped at the corpus
    ("rescore_below_candidates", expect(10, 100, 100, 0.7, 0, 0, 0)),  # rescore raised to candidates
    ("rescore_without_store", expect(10, 100, 0, 0.7, 0, 0, 0)),
    ("rescore_over_corpus", expect(10, 100, 1000, 0.7, 0, 0, 0)),
    ("config_rescore_graph", expect(10, 100, 300, 0.7, 0, 1, 2)),
    ("weight_clamp_hybrid", expect(10, 100, 0, 1.0, 1, 1, 1)),
    ("hybrid_without_index", expect(10, 100, 0, 1.0, 0, 1, 1)),
])
def test_option_resolution(rules, name, want):
    assert resolved(rules, name) == want


def test_invalid_top_k_throws(rules):
    assert "zero_topk invalid_argument" in rules


def test_lexical_terms_drop_markers_negatives_and_repeats(rules):
    terms = [l for l in rules if l.startswith("terms")]
    assert terms[0] == "terms 7 9 3"
    assert terms[1] == "terms" and terms[2] == "terms 5" and terms[3] == "terms"
    assert "terms_capped 1 2 3" in rules


def test_allow_mask(rules):
    assert "mask 1 0 0 1 0 0 0 0 0 1" in rules
    assert "mask_empty 0" in rules
