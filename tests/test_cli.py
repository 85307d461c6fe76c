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
