"""CPU tier: the C++ JSON config loader (include/zcgvs/engine/config_loader.hpp) against the
reference's own loader.

tests/golden/configs.json holds the reference's four configs (configs/*.json) and the fields its
python/zcgvs_tools/config.py (config_from_dict / config_from_json, run unchanged by
tests/golden/make_configs.py) makes of them, its errors for an unknown key and an unknown
metric, and its path resolution on a small directory tree. A driver compiled here
(tests/cpp/config_search.cpp) loads the same texts with the C++ loader; every field must match.
"""

from __future__ import annotations

import json
import os
import shutil
import subprocess

import pytest

from conftest import PKG, ROOT

GOLDEN = json.loads((ROOT / "tests" / "golden" / "configs.json").read_text())


@pytest.fixture(scope="module")
def driver(zc, tmp_path_factory):
    exe = tmp_path_factory.mktemp("cpp") / "config_search"
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cxx = shutil.which("g++") or shutil.which("c++")
    cmd = [cxx, "-std=c++17", "-O2", f"-I{ROOT / 'include'}", f"-I{cuda}/include",
           str(ROOT / "tests/cpp/config_search.cpp"), "-o", str(exe), f"-L{PKG}", "-lzcgvs_sm100",
           f"-L{cuda}/lib64", "-lcudart", f"-Wl,-rpath,{PKG}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def _fields(stdout: str) -> dict:
    return dict(line.split("=", 1) for line in stdout.splitlines() if "=" in line)


def _as_text(value) -> str:
    if isinstance(value, bool):
        return "1" if value else "0"
    if isinstance(value, float):
        return f"{value:.9g}" if value != int(value) else f"{value:.9g}"
    return str(value)


def _run(driver, *args, cwd=None):
    return subprocess.run([str(driver), *args], capture_output=True, text=True, timeout=60, cwd=cwd)


@pytest.mark.parametrize("name", sorted(GOLDEN["configs"]))
def test_reference_configs_load_to_the_reference_fields(driver, tmp_path, name):
    case = GOLDEN["configs"][name]
    path = tmp_path / name
    path.write_text(case["text"])
    res = _run(driver, f"dump={path}")
    assert res.returncode == 0, res.stderr
    got = _fields(res.stdout)
    for key, value in case["fields"].items():
        want = _as_text(value) if key != "dense_weight" else f"{float(value):.9g}"
        if key == "dense_weight":
            # float field: the C++ float of the JSON number (the reference stores a C++ float too)
            assert abs(float(got[key]) - float(value)) < 1e-7, key
        else:
            assert got[key] == want, f"{name}: {key} = {got[key]!r}, reference {want!r}"


@pytest.mark.parametrize("case", ["unknown_key", "unknown_metric"])
def test_errors_match_the_reference(driver, tmp_path, case):
    path = tmp_path / "bad.json"
    path.write_text(GOLDEN[case]["text"])
    res = _run(driver, f"dump={path}")
    assert res.returncode == 2
    assert GOLDEN[case]["error"] in res.stderr


def test_metric_names(driver, tmp_path):
    for name, want in GOLDEN["metric_names"].items():
        path = tmp_path / "m.json"
        path.write_text(json.dumps({"metric": name}))
        res = _run(driver, f"dump={path}")
        assert res.returncode == 0 and _fields(res.stdout)["metric"] == want, name


def test_paths_resolve_against_the_search_roots_like_the_reference(driver, tmp_path):
    case = GOLDEN["paths"]
    root = tmp_path / "tree"
    for rel in case["tree"]:
        (root / rel).parent.mkdir(parents=True, exist_ok=True)
        (root / rel).write_bytes(b"")
    config = root / case["config"]
    config.write_text(case["text"].replace("<root>", str(root)))
    res = _run(driver, f"file={config}", cwd=root / case["cwd"])
    assert res.returncode == 0, res.stderr
    got = _fields(res.stdout)
    for key, value in case["fields"].items():
        assert got[key].replace(str(root), "<root>") == value, key


def test_type_errors_and_malformed_json_are_rejected(driver, tmp_path):
    for text, expect in ((json.dumps({"default_top_k": 2.5}), "needs an integer"),
                         (json.dumps({"hybrid": "yes"}), "true or false"),
                         (json.dumps({"embeddings_path": 3}), "needs a string"),
                         ('{"metric": "cosine",}', "invalid JSON"),
                         ("[1, 2]", "must be a JSON object")):
        path = tmp_path / "t.json"
        path.write_text(text)
        res = _run(driver, f"dump={path}")
        assert res.returncode == 2 and expect in res.stderr, (text, res.stderr)


def test_json_strings_with_escapes(driver, tmp_path):
    path = tmp_path / "e.json"
    path.write_text('{"encoder_output_name": "a\\"b\\\\c\\u00e9\\ud83d\\ude00\\n", "dense_weight": 1e-1}')
    res = _run(driver, f"dump={path}")
    assert res.returncode == 0, res.stderr
    assert _fields(res.stdout)["encoder_output_name"] == 'a"b\\cé😀'
    assert abs(float(_fields(res.stdout)["dense_weight"]) - 0.1) < 1e-7
