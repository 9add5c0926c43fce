"""The Node-API addon (gemma4_cuda.node, napi/g4_napi.c) through a minimal Node-API host
(tests/napi_host/node_host.c) that implements the calls the addon makes, since Node.js is not
installed: registration as Node performs it, argument checking, C-ABI errors surfacing as thrown
errors with a G4_ERR_* code, and (on a GPU) a generation through createContext / initRandom /
prefill / decodeAhead / verify equal to the oracle's greedy tokens."""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

import __graft_entry__ as entry

ROOT = Path(__file__).resolve().parent.parent
SEED = 0x6E6D6134


@pytest.fixture(scope="module")
def host(tmp_path_factory, pkg):
    bl = entry._load_build_lib()
    addon = bl.build_napi()
    exe = tmp_path_factory.mktemp("napi") / "node_host"
    subprocess.run(["gcc", "-O1", "-std=gnu11", "-rdynamic", "-o", str(exe),
                    str(ROOT / "tests" / "napi_host" / "node_host.c"), "-ldl"], check=True)
    return exe, addon


def run(host, *args):
    exe, addon = host
    r = subprocess.run([str(exe), str(addon), *map(str, args)], capture_output=True, text=True, timeout=600)
    return r.returncode, r.stdout


def test_addon_registers_every_export(host):
    rc, out = run(host, "exports")
    assert rc == 0, out
    names = {line.split()[1] for line in out.splitlines() if line.startswith("export ")}
    assert names == {"createContext", "destroyContext", "initRandom", "uploadWeight", "setScalar",
                     "prefill", "decode", "decodeAhead", "verify", "decodeBatch", "kvTruncate",
                     "readLogits", "version"}
    assert "version gemma4_cuda" in out


def test_addon_errors_are_thrown_with_codes(host):
    rc, out = run(host, "errors")
    assert rc == 0, out
    lines = [l for l in out.splitlines() if l.startswith("threw")]
    assert len(lines) == 4, out
    assert lines[0].startswith("threw G4_ERR_CUDA: CUDA device 99 is not available")
    assert lines[1].startswith("threw G4_ERR_INVALID: createContext(device, options?)")
    assert lines[2].startswith("threw G4_ERR_INVALID: prefill(")
    assert lines[3].startswith("threw G4_ERR_INVALID: decode(")


@pytest.mark.gpu
def test_addon_generation_matches_oracle(host, pkg, O, cuda):
    a = entry.tiny_arch(pkg)
    opts = dict(layerCount=a.layer_count, hiddenSize=a.hidden_size, globalLayerMask=a.global_layer_mask,
                slidingWindow=a.sliding_window, kvProducerLayers=a.kv_producer_layers,
                producerIntermediate=a.producer_intermediate, consumerIntermediate=a.consumer_intermediate,
                vocabSize=a.vocab_size, maxSeqs=1, maxContext=64, maxStepColumns=16)
    prompt = [int(t) for t in O.synth_prompt(SEED, 12, a.vocab_size)]
    rc, out = run(host, "generate", *[f"{k}={v}" for k, v in opts.items()], "--", SEED, 6, *prompt)
    assert rc == 0, out
    want, _ = O.Model(SEED, entry.oracle_arch(O, a)).generate(prompt, 6, 64)
    toks = [int(x) for x in out.splitlines()[0].split()[1:]]
    assert toks == [int(t) for t in want]
    ver = [int(x) for x in out.splitlines()[1].split()[1:]]
    assert ver == toks[1:5]
    threw = [l for l in out.splitlines() if l.startswith("threw")]
    assert threw[0].startswith("threw G4_ERR_INVALID: token id -5 outside the vocabulary")
    assert threw[1].startswith("threw G4_ERR_INVALID: decode(")
