"""The reference's own command-line program (src/main.c, unmodified) on the B200
engine: `oracle/_ref/qwen-b200` is main.c + the reference tokenizer linked
against libqwenb200 (oracle/Makefile target relink-cli), `oracle/_ref/qwen-ref`
the same main.c on the reference engine (target reference-cli).  Both run on a
4-layer model whose GGUF carries a byte-level tokenizer vocabulary; the text
they generate must be the same, character for character, in the speculative
loop (src/main.c:158-225) and in the sampler loop at temperature 0
(src/main.c:232-248, sampler_sample's greedy branch).  The reference's SSE
server (server.py) streams exactly this standard output from the binary it
spawns, so it serves the B200 engine once that binary is `qwen-b200`.
"""
import os
import subprocess

import pytest

from conftest import ROOT, qb

pytestmark = pytest.mark.gpu

B200_CLI = os.path.join(ROOT, "oracle", "_ref", "qwen-b200")
REF_CLI = os.path.join(ROOT, "oracle", "_ref", "qwen-ref")
have = pytest.mark.skipif(not (os.path.exists(B200_CLI) and os.path.exists(REF_CLI)),
                          reason="the CLI binaries are built with the reference sources (make -C oracle relink-cli "
                                 "reference-cli)")


def generation(binary, gguf, prompt, n, spec, temp="0"):
    out = subprocess.run([binary, "-m", gguf, "-p", prompt, "-n", str(n), "-c", "512", "-t", "4", "--spec",
                          str(spec), "--temp", temp], capture_output=True, text=True, timeout=600,
                         errors="replace")
    assert out.returncode == 0, (binary, out.returncode, out.stderr[-2000:])
    text = out.stdout
    assert "Generation: " in text, text[-2000:]
    body = text.split("Generation: ", 1)[1]
    return body.split("\n================================================", 1)[0]


@pytest.fixture(scope="module", params=[0, 1], ids=["tiny", "tiny_mixed"])
def tok_gguf(request, workdir):
    path = os.path.join(workdir, f"tiny_tok_{request.param}.gguf")
    if not os.path.exists(path):
        qb.write_synth_gguf(path, qb.TINY, seed=11, profile=request.param, tokenizer=1)
    return path


@have
@pytest.mark.parametrize("spec", [1, 3, 0])
@pytest.mark.parametrize("prompt", ["The quick brown fox", "in the heart of the matter, 2 + 2 = 4"])
def test_reference_cli_on_b200_prints_the_reference_text(tok_gguf, spec, prompt):
    want = generation(REF_CLI, tok_gguf, prompt, 40, spec)
    got = generation(B200_CLI, tok_gguf, prompt, 40, spec)
    assert got == want
    assert len(want) > 40   # 40 tokens of text came out
