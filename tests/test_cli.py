"""llama_generate program: argument handling that needs no GPU."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "asicfortranai_b200", "bin", "llama_generate")


@pytest.fixture(scope="module")
def cli():
    from asicfortranai_b200 import build
    build.build()
    assert os.access(CLI, os.X_OK)
    return CLI


def test_help_lists_the_serving_flags(cli):
    r = subprocess.run([cli, "--help"], capture_output=True, text=True)
    assert r.returncode == 0
    for flag in ("--prompt", "--max-tokens", "--temperature", "--json", "--weights", "--tokens-in"):
        assert flag in r.stdout


def test_bad_arguments_exit_2(cli, tmp_path):
    assert subprocess.run([cli, "--bogus"], capture_output=True).returncode == 2
    assert subprocess.run([cli, "--max-tokens"], capture_output=True).returncode == 2
    assert subprocess.run([cli, "--format", "int7"], capture_output=True).returncode == 2
    bad = tmp_path / "tokens.bin"
    bad.write_bytes(np.array([5, 1, 2], np.int32).tobytes())          # count 5, only 2 ids
    r = subprocess.run([cli, "--tokens-in", str(bad)], capture_output=True, text=True)
    assert r.returncode == 2 and "cannot read token ids" in r.stderr


def test_environment_defaults_are_read(cli):
    env = dict(os.environ, LLAMA_GENERATE_MODEL="no-such-model")
    r = subprocess.run([cli, "--prompt", "x"], capture_output=True, text=True, env=env)
    assert r.returncode == 2 and "unknown model no-such-model" in r.stderr
    # a flag overrides the environment's choice before any device work
    r = subprocess.run([cli, "--model", "also-missing"], capture_output=True, text=True, env=env)
    assert r.returncode == 2 and "unknown model also-missing" in r.stderr


FAKE_TOKENIZER = r"""
import sys
import numpy as np
mode, src, dst = sys.argv[1:4]
open(sys.argv[0] + ".log", "a").write(mode + "\n" + open(src, "rb").read().decode("latin-1") + "\n--\n")
if mode == "encode":
    np.array([3, 5, 6, 7], np.int32).tofile(dst)
else:
    open(dst, "w").write("decoded")
"""


def _run_tokenizer_phase(cli, tmp_path, tokenizer, *extra, stdin=""):
    # the tiny shape and one new token: harmless where a GPU is present; on a host without
    # one the program stops at the device context, after the prompt and token steps
    return subprocess.run([cli, "--model", "tiny", "--max-tokens", "1", *extra] +
                          (["--tokenizer", tokenizer] if tokenizer else []),
                          capture_output=True, text=True, input=stdin, timeout=300)


def test_tokenizer_protocol(cli, tmp_path):
    """llama_generate.f90:162-214: the prompt goes to `<cmd> encode prompt.txt tokens.bin`
    as a text line and comes back as an int32 count followed by the int32 ids."""
    import sys
    tok = tmp_path / "tok.py"
    tok.write_text(FAKE_TOKENIZER)
    r = _run_tokenizer_phase(cli, tmp_path, f"{sys.executable} {tok}", "--prompt", "hello 'quoted' world")
    assert " Prompt tokens: 3" in r.stdout, r.stdout + r.stderr
    log = (tmp_path / "tok.py.log").read_text()
    assert log.startswith("encode\nhello 'quoted' world\n")


def test_tokenizer_failure_falls_back_to_placeholder_ids(cli, tmp_path):
    """:181-186 -- a failing tokenizer leaves the placeholder ids 1..10."""
    r = _run_tokenizer_phase(cli, tmp_path, "false", "--prompt", "x")
    assert "Tokenizer failed, using placeholder tokens" in r.stderr
    assert " Prompt tokens: 10" in r.stdout


def test_empty_stdin_uses_the_default_prompt(cli, tmp_path):
    """:39-44 -- an empty prompt line from stdin selects the default prompt."""
    r = _run_tokenizer_phase(cli, tmp_path, None, stdin="\n")
    assert "Using default prompt: Explain quantum computing in simple terms:" in r.stdout
    assert " Prompt tokens: 10" in r.stdout


def test_scratch_directory_removed_on_early_exit(cli, tmp_path):
    """The tokenizer's scratch directory goes away on every exit path (here: the device
    step fails on a host without a GPU, or the run completes where there is one)."""
    import glob
    import sys
    tok = tmp_path / "tok.py"
    tok.write_text(FAKE_TOKENIZER)
    before = set(glob.glob("/tmp/llama_generate_*"))
    _run_tokenizer_phase(cli, tmp_path, f"{sys.executable} {tok}", "--prompt", "x")
    _run_tokenizer_phase(cli, tmp_path, "false", "--prompt", "y")
    assert set(glob.glob("/tmp/llama_generate_*")) <= before
