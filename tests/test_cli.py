"""The `jalapeno` command line against the reference's engine/src/main.rs:
argument checks, messages and exit status (host only), then greedy,
speculative and --time-rows runs on checkpoints written to disk (GPU)."""
import json
import os
import subprocess
from pathlib import Path

import pytest

import checkpoint as CK
import oracle as O

PKG = Path(__file__).resolve().parents[1] / "jalapenos-at-home_b200"
CLI = PKG / "bin" / "jalapeno"
USAGE = ("usage: engine <cpu|metal|gpu> <model> <new tokens> [--draft <model>] [--gamma <count>] [--mxfp4] "
         "[--adaptive] [--max-gamma <count>] [--prefill-backend <cpu|metal|gpu>] [--draft-backend "
         "<cpu|metal|gpu>] [--stats] < prompt.json")


@pytest.fixture(scope="module")
def cli():
    if not CLI.exists():
        subprocess.run(["make", "-C", str(PKG), "bin/jalapeno"], check=True)
    return CLI


def run(cli, args, prompt="[1, 2, 3]", env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([str(cli), *args], input=prompt, capture_output=True, text=True, env=e, timeout=600)


def expect_error(cli, args, message, prompt="[1, 2, 3]", env=None):
    r = run(cli, args, prompt, env)
    assert r.returncode == 1, r
    assert r.stderr.strip() == "Error: " + message, r.stderr
    assert r.stdout == ""


# main.rs:9-14: the first argument selects the backend, anything else is a usage error
@pytest.mark.parametrize("args", [[], ["tpu", "m", "3"]])
def test_usage(cli, args):
    expect_error(cli, args, json.dumps(USAGE))


@pytest.mark.parametrize("args,message", [
    (["gpu"], '"missing model"'),                                   # main.rs:15
    (["gpu", "m"], '"missing token count"'),                        # main.rs:16
    (["gpu", "m", "x3"], "ParseIntError { kind: InvalidDigit }"),
    (["gpu", "m", ""], "ParseIntError { kind: Empty }"),
    (["gpu", "m", "3", "--gamma"], '"missing gamma"'),
    (["gpu", "m", "3", "--gamma", "0"], '"gamma must be positive"'),  # main.rs:43-45
    (["gpu", "m", "3", "--max-gamma"], '"missing max gamma"'),
    (["gpu", "m", "3", "--draft"], '"missing draft model"'),
    (["gpu", "m", "3", "--time-rows"], '"missing row counts"'),
    (["gpu", "m", "3", "--prefill-backend", "tpu"], '"backend must be cpu, metal or gpu"'),
    (["gpu", "m", "3", "--draft-backend"], '"missing draft backend"'),
    (["gpu", "m", "3", "--verbose"], '"unexpected argument: --verbose"'),
    (["gpu", "m", "3", "--stats"], '"--adaptive, --draft-backend and --stats require --draft"'),
    (["gpu", "m", "3", "--adaptive"], '"--adaptive, --draft-backend and --stats require --draft"'),
    (["gpu", "m", "3", "--draft-backend", "gpu"], '"--adaptive, --draft-backend and --stats require --draft"'),
    (["gpu", "m", "3", "--draft", "d", "--adaptive", "--gamma", "9"],
     '"adaptive gamma must be positive and no greater than max gamma"'),  # scheduler.rs:18-22
])
def test_argument_errors(cli, args, message):
    expect_error(cli, args, message)


def test_prompt_errors(cli):
    expect_error(cli, ["gpu", "m", "3"], '"prompt is empty"', prompt="[]")  # main.rs:56-58
    for bad in ("", "{}", "[1, 2.5]", "[1, -2]", "[1 2]", "[1, 2] 3", "[1,"):
        r = run(cli, ["gpu", "m", "3"], prompt=bad)
        assert r.returncode == 1 and r.stderr.startswith("Error: Error("), (bad, r.stderr)


def test_backends_without_a_gpu_engine(cli):
    # model.rs:64-68: a gpu model needs a gpu prefill; cpu and metal are not built here
    expect_error(cli, ["gpu", "m", "3", "--prefill-backend", "cpu"],
                 '"the gpu backend keeps the KV cache on the GPU, so prefill must use gpu too"')
    expect_error(cli, ["metal", "m", "3"], '"the metal backend is not part of this build: use gpu"')


def test_missing_model_directory(cli, tmp_path):
    r = run(cli, ["gpu", "nothing", "3"], env={"JALAPENO_WEIGHTS": str(tmp_path)})
    assert r.returncode == 1 and "config.json" in r.stderr, r.stderr


@pytest.fixture(scope="module")
def weights(tmp_path_factory):
    """weights/tiny, weights/tiny-draft and their -MXFP4 variants."""
    root = tmp_path_factory.mktemp("weights")
    for name, seed in (("tiny", 0), ("tiny-draft", 1)):
        CK.write_model(O.Model.synthetic(name, seed), root / name, quantized=False)
        CK.write_model(O.Model.synthetic(name, seed, mxfp4=True), root / (name + "-MXFP4"), quantized=True)
    return root


@pytest.mark.gpu
@pytest.mark.parametrize("mxfp4", [False, True])
def test_greedy_and_speculative(cli, weights, mxfp4):
    import jalapeno as J

    prompt = O.prompt_ids(12, 1000, 2)
    env = {"JALAPENO_WEIGHTS": str(weights)}
    flag = ["--mxfp4"] if mxfp4 else []
    r = run(cli, ["gpu", "tiny", "10", *flag], json.dumps(prompt), env)
    assert r.returncode == 0, r.stderr
    greedy = json.loads(r.stdout)
    m = J.Model.load(weights / ("tiny-MXFP4" if mxfp4 else "tiny"))
    assert greedy == m.generate(prompt, 10)[len(prompt):]

    # main.rs:72-109: generate_scheduled, stats on stderr, the same tokens on stdout
    r = run(cli, ["gpu", "tiny", "10", "--draft", "tiny-draft", "--gamma", "3", "--adaptive", "--stats", *flag],
            json.dumps(prompt), env)
    assert r.returncode == 0, r.stderr
    assert json.loads(r.stdout) == greedy
    lines = r.stderr.strip().splitlines()
    stats = json.loads(lines[0])
    assert list(stats) == sorted(stats)
    assert set(stats) == {"adaptive", "elapsed_ms", "generated", "accepted", "drafted", "rounds",
                          "target_prefill_backend", "draft_prefill_backend", "draft_backend", "verify_backend",
                          "prefill", "draft", "verify", "round_stats"}
    assert stats["adaptive"] is True and stats["generated"] == 10
    assert stats["verify_backend"] == stats["draft_backend"] == "gpu"
    assert len(stats["round_stats"]) == stats["rounds"]
    assert sum(s["accepted"] for s in stats["round_stats"]) == stats["accepted"]
    assert stats["verify"]["passes"] >= stats["rounds"] and stats["prefill"]["passes"] >= 2
    assert lines[1] == "accepted %d / %d draft tokens in %d rounds" % (
        stats["accepted"], stats["drafted"], stats["rounds"])


@pytest.mark.gpu
def test_time_rows(cli, weights):
    r = run(cli, ["gpu", "tiny", "4", "--time-rows", "1,3"], json.dumps(O.prompt_ids(8, 1000, 2)),
            {"JALAPENO_WEIGHTS": str(weights)})
    assert r.returncode == 0, r.stderr
    rows = [json.loads(line) for line in r.stdout.strip().splitlines()]
    assert [x["rows"] for x in rows] == [1, 3]
    assert all(x["gpu_ms"] > 0 and x["wall_ms"] > 0 and list(x) == sorted(x) for x in rows)
