"""llama_generate program on the GPU: its tokens equal the oracle's generation over the
same checkpoint, for the reference's greedy and nucleus paths and for the serving API's
exact invocation."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from asicfortranai_b200 import weight_files as wf
from oracle import oracle as orc
from tests.model_util import TINY, make_weights

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "asicfortranai_b200", "bin", "llama_generate")


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("ckpt")
    w = make_weights(TINY, seed=11)
    wf.write_safetensors(d / "m.safetensors", wf.llama_3p5bit_tensors(TINY, w, float_dtype=np.float32))
    return d / "m.safetensors", w


def _ids_file(path, ids):
    path.write_bytes(np.array([len(ids), *ids], np.int32).tobytes())


def _run(args, env=None):
    r = subprocess.run([CLI, *args], capture_output=True, text=True, timeout=300,
                       env=dict(os.environ, **(env or {})))
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_greedy_tokens_match_oracle(ckpt, tmp_path):
    path, w = ckpt
    prompt = orc.gen_tokens(8, 12, 1, TINY["vocab"])
    _ids_file(tmp_path / "in.bin", prompt)
    out = _run(["--model", "tiny", "--weights", str(path), "--tokens-in", str(tmp_path / "in.bin"),
                "--max-tokens", "20", "--temperature", "0", "--json", "--no-eos",
                "--tokens-out", str(tmp_path / "out.bin")])
    want = orc.OracleModel(TINY, w).generate(prompt, 20)
    assert out["token_ids"] == [int(x) for x in want] and out["tokens"] == 20 and out["prompt_tokens"] == 8
    got = np.fromfile(tmp_path / "out.bin", np.int32)
    assert got[0] == 28 and list(got[1:9]) == list(prompt) and list(got[9:]) == list(want)


def test_nucleus_sampling_matches_oracle(ckpt, tmp_path):
    path, w = ckpt
    prompt = orc.gen_tokens(6, 12, 2, TINY["vocab"])
    _ids_file(tmp_path / "in.bin", prompt)
    out = _run(["--model", "tiny", "--weights", str(path), "--tokens-in", str(tmp_path / "in.bin"),
                "--max-tokens", "24", "--temperature", "0.8", "--seed", "7", "--json", "--no-eos"])
    want = orc.OracleModel(TINY, w).generate(prompt, 24, sampling=dict(mode=3, top_p=0.95, seed=7), seq=0)
    assert out["token_ids"] == [int(x) for x in want]


def test_serving_api_invocation(ckpt, tmp_path):
    """api/inference_api.py:464-477: --prompt P --max-tokens N --temperature T --json; the
    model comes from the environment; no tokenizer -> placeholder prompt ids 1..10."""
    path, w = ckpt
    out = _run(["--prompt", "What is a bond?", "--max-tokens", "12", "--temperature", "0.0", "--json"],
               env={"LLAMA_GENERATE_MODEL": "tiny", "LLAMA_GENERATE_WEIGHTS": str(path)})
    want = orc.OracleModel(TINY, w).generate(np.arange(1, 11, dtype=np.int32), 12, stop_at_eos=True)
    assert out["prompt_tokens"] == 10
    assert out["tokens"] == len(want) and out["token_ids"] == [int(x) for x in want]
    assert out["text"] == " ".join(str(int(x)) for x in want)


def test_tokenizer_command_round_trip(ckpt, tmp_path):
    """The tokenizer protocol of llama_generate.f90:162-253 with a stand-in tokenizer:
    bytes of the prompt -> ids (byte + 3), ids -> text."""
    path, w = ckpt
    tok = tmp_path / "tok.py"
    tok.write_text(
        "import sys, struct\n"
        "mode, src, dst = sys.argv[1:4]\n"
        "if mode == 'encode':\n"
        "    b = open(src, 'rb').read().strip()\n"
        "    ids = [c + 3 for c in b]\n"
        "    open(dst, 'wb').write(struct.pack('i', len(ids)) + struct.pack(f'{len(ids)}i', *ids))\n"
        "else:\n"
        "    d = open(src, 'rb').read(); n = struct.unpack('i', d[:4])[0]\n"
        "    ids = struct.unpack(f'{n}i', d[4:4 + 4 * n])\n"
        "    open(dst, 'w').write('|'.join(map(str, ids)) + '\\n')\n")
    out = _run(["--model", "tiny", "--weights", str(path), "--prompt", "hi!", "--max-tokens", "5",
                "--temperature", "0", "--json", "--no-eos", "--tokenizer", f"{sys.executable} {tok}"])
    prompt = np.array([ord(c) + 3 for c in "hi!"], np.int32)
    want = orc.OracleModel(TINY, w).generate(prompt, 5)
    assert out["prompt_tokens"] == 3 and out["token_ids"] == [int(x) for x in want]
    assert out["text"] == "|".join(str(int(x)) for x in [*prompt, *want])
