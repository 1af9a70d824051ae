"""Generates tests/golden/configs.json from the reference's own config loader: its JSON configs
(configs/*.json) and what its python/zcgvs_tools/config.py makes of them. Run where the
reference tree exists (its path in ZCGVS_REFERENCE):

    ZCGVS_REFERENCE=<reference checkout> python tests/golden/make_configs.py

config.py imports the reference's compiled pybind module (zcgvs_engine) only for its
EngineConfig / Metric / SimilarityBackend types; that module is not built here, so a stand-in
module with the same attribute names and the defaults of include/zcgvs/engine/engine_config.hpp
is installed first. Everything else (unknown-key rejection, metric and backend names, path
resolution against the search roots) is the reference's code running unchanged. The fixture
stores each config's text and resulting fields, the errors of an unknown key and an unknown
metric, and a path-resolution case on a small directory tree (paths relative to its root).
"""

from __future__ import annotations

import enum
import json
import os
import sys
import tempfile
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent
if not os.environ.get("ZCGVS_REFERENCE"):
    sys.exit("set ZCGVS_REFERENCE to the reference checkout (the script imports its Python tools)")
REF = Path(os.environ["ZCGVS_REFERENCE"])


class Metric(enum.Enum):
    Cosine = 0
    DotProduct = 1
    L2 = 2


class SimilarityBackend(enum.Enum):
    Custom = 0
    Cublas = 1


class EngineConfig:
    """Stand-in for the pybind EngineConfig: the fields and defaults of engine_config.hpp."""

    def __init__(self):
        self.embeddings_path = ""
        self.metadata_path = ""
        self.vocab_path = ""
        self.rescore_embeddings_path = ""
        self.lexical_index_path = ""
        self.encoder_model_path = ""
        self.encoder_output_name = "last_hidden_state"
        self.encoder_max_seq_len = 256
        self.reranker_backend = "onnx"
        self.reranker_model_path = ""
        self.reranker_output_name = "logits"
        self.reranker_max_seq_len = 256
        self.reranker_batch_size = 32
        self.device_id = 0
        self.lowercase = True
        self.metric = Metric.Cosine
        self.similarity_backend = SimilarityBackend.Custom
        self.default_top_k = 10
        self.default_candidates = 100
        self.rescore_candidates = 0
        self.hybrid = False
        self.dense_weight = 0.7
        self.max_query_terms = 64
        self.use_cuda_graphs = False


def fields(config: EngineConfig) -> dict:
    out = dict(vars(config))
    out["metric"] = config.metric.name
    out["similarity_backend"] = config.similarity_backend.name
    return out


def main() -> None:
    stand_in = types.ModuleType("zcgvs_engine")
    stand_in.Metric, stand_in.SimilarityBackend, stand_in.EngineConfig = Metric, SimilarityBackend, EngineConfig
    sys.modules["zcgvs_engine"] = stand_in
    sys.path.insert(0, str(REF / "python"))
    from zcgvs_tools import config as ref_config

    out: dict = {"configs": {}}
    for path in sorted((REF / "configs").glob("*.json")):
        text = path.read_text()
        out["configs"][path.name] = {"text": text, "fields": fields(ref_config.config_from_dict(json.loads(text)))}

    def error_of(values: dict) -> str:
        try:
            ref_config.config_from_dict(values)
        except (KeyError, ValueError) as error:
            return error.args[0]
        raise AssertionError("expected an error")

    out["unknown_key"] = {"text": json.dumps({"metric": "dot", "bogus_field": 1}),
                          "error": error_of({"metric": "dot", "bogus_field": 1})}
    out["unknown_metric"] = {"text": json.dumps({"metric": "hamming"}), "error": error_of({"metric": "hamming"})}
    out["metric_names"] = {name: ref_config.metric_from_name(name).name
                           for name in ("cosine", "COSINE", "dot", "DotProduct", "ip", "l2", "Euclidean")}

    # Path resolution: a config under <root>/configs naming files found beside it, under the root,
    # nowhere, and by an absolute path; run from a directory that holds none of them.
    with tempfile.TemporaryDirectory() as tmp:
        root = Path(tmp).resolve()
        tree = ["configs/local.meta", "data/corpus.bin", "data/corpus.lex", "elsewhere/.keep"]
        for rel in tree:
            (root / rel).parent.mkdir(parents=True, exist_ok=True)
            (root / rel).write_bytes(b"")
        values = {"embeddings_path": "data/corpus.bin", "metadata_path": "local.meta",
                  "lexical_index_path": "data/corpus.lex", "vocab_path": "models/missing.txt",
                  "rescore_embeddings_path": "<root>/data/corpus.bin", "encoder_model_path": ""}
        text = json.dumps(values).replace("<root>", str(root))
        (root / "configs" / "c.json").write_text(text)
        cwd = os.getcwd()
        os.chdir(root / "elsewhere")
        try:
            resolved = fields(ref_config.config_from_json(root / "configs" / "c.json"))
        finally:
            os.chdir(cwd)
        out["paths"] = {
            "tree": tree,
            "config": "configs/c.json",
            "text": json.dumps(values),
            "cwd": "elsewhere",
            "fields": {k: resolved[k].replace(str(root), "<root>") for k in values},
        }
    (HERE / "configs.json").write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
    print("configs.json", (HERE / "configs.json").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
