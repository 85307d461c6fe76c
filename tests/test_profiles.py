"""The profile summaries name commands that run committed files only: every `python X`
they cite is a tracked file outside the working-files folder, every option it passes to
bench.py exists, and every ncu command leaves the clocks alone (--clock-control none)."""
import glob
import os
import re
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _commands():
    out = []
    for p in sorted(glob.glob(os.path.join(ROOT, "profiles", "*.md"))):
        text = open(p).read().replace("\\\n", " ")
        for line in text.splitlines():
            line = line.strip().strip("`")
            if re.match(r"(python \S+\.py|ncu -)", line):
                out.append((os.path.basename(p), line))
    return out


def test_every_profile_names_a_command():
    names = {os.path.basename(p) for p in glob.glob(os.path.join(ROOT, "profiles", "*.md"))}
    assert names and names == {n for n, _ in _commands()}


def test_commands_run_committed_files_with_known_options():
    tracked = set(subprocess.run(["git", "ls-files"], cwd=ROOT, capture_output=True, text=True).stdout.split())
    bench_help = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--help"], cwd=ROOT,
                                capture_output=True, text=True, timeout=120).stdout
    for name, cmd in _commands():
        if cmd.startswith("ncu "):
            assert "--clock-control none" in cmd, (name, cmd)
        for m in re.finditer(r"python (\S+\.py)((?: [^|&;]*)?)", cmd):
            script, args = m.group(1), m.group(2)
            assert script in tracked and not script.startswith("_work"), (name, script)
            if script == "bench.py":
                for opt in re.findall(r"(--[a-z][a-z-]*)", args):
                    assert opt in bench_help, (name, opt)
