"""Weight-space experiment bench: edit a model's weights along a residual direction and measure
the effect on a small, fixed, resumable GSM8K / MATH development run, with provenance checks at
every step. This is the counterpart of the reference's `tools/weight-space/` bench, re-targeted
from llama.cpp / GGUF to this framework's own engine and safetensors checkpoints:

  prepare       `bench.py prepare`      GSM8K-train mini dev/validation split (from a local JSONL)
                `prepare_math.py`       MATH-train level 4/5 integer-answer subset (local parquet)
  audit         `split_audit.py`        lexical dev/validation overlap audit
  serve         `server.py`             loopback completion server over the block-diffusion decoder
  run           `launch.py`             start the server, run the bench, stop only that server
                `bench.py run`          resumable run against a loopback server (manifest + JSONL)
  compare       `bench.py compare`      paired accuracy delta, bootstrap interval, exact McNemar
  collect       `collect.py`            verified bundle of completed runs under a comparison plan
  uncertainty   `uncertainty.py`        binomial-tail win/loss intervals, Bonferroni paired bound
  capture       `native_tools/bin/capture` + `capture_data.py`   residual vectors per prompt/layer
  derive        `derive_direction.py`   one gated residual direction from early/late probe pairs
  edit          `surgery.py`            W <- W - s d (d^T W) on MLP down projections of a copy,
                                        bytes outside the edited tensors verified unchanged
  score         `symbolic_score.py`     boxed-answer scorer, `symbolic_process.py` bounded worker
  claim         `controller_claim.py`   exclusive ownership receipt for an output directory

Every writer creates new files exclusively (no silent overwrite); every reader re-verifies the
SHA-256 digests it was given.
"""
