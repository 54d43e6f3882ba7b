"""The drop-in check: vkllm.c's OWN test programs, compiled unchanged against this repository's
include/ and linked to libvkllm_b200.so, run on the B200.

oracle/refpin/Makefile builds them from the reference checkout (only where it exists; they travel
as built binaries under oracle/_ref/compat/). Their "src/core/..." and "src/models/..." includes
resolve to include/, and oracle/refpin/stub/check.h stands in for libcheck (the unit-test library
they are written against). Each op program draws random inputs with rand(), runs the op through
the C API (tensor_new, commands upload/submit/wait, vkllm_op_*_init/run/post_run, download) and
compares with its own in-file CPU function under its own tolerance:

  tests/vkllm_test_op_{add,arg_max,bin,copy,embedding,ffn_up_and_gate,matmul,permute,rmsnorm,rope,
  softmax,update_rows}.c, tests/vkllm_test_tensor_reshape.c, tests/vkllm_test_hashmap.c

tests/vkllm_test_infer_gguf.c is the reference's token loop: load a GGUF, tokenize a fixed prompt,
then per token tensor_new / graph_new / build_graph / init / upload / run / post_run / read the
mapped argmax / graph_free, printing the generated pieces. It runs here on the tiny synthetic GGUF
(whose vocabulary pieces are "<tN>", so the printed text gives the token ids back), and its tokens
must equal the CPU oracle's greedy tokens from the same prompt ids for the first 32 steps.

Three outcomes are the reference's own, not this library's, and the checks below name them exactly:
  * vkllm_test_op_arg_max compares the GPU with a first-maximum CPU function, while the reference's
    shader breaks ties by its lane/tree rule (src/shaders/vkllm_arg_max.comp:54-90), which this
    library keeps. With fp16 inputs in [-1000, 1000] equal maxima occur; a mismatch is accepted
    only where the two indices hold the same value.
  * vkllm_test_tensor_reshape's table has three "valid" cases whose element counts differ
    (entries 4, 8 and 13: [4,8,64,64] -> [1,1,1024,256] twice, [8,16,128,64] -> [2,64,256,64]); the
    program's own count check fails there before any library call.
  * vkllm_test_infer_gguf returns its last vkllm_err_t, and VKLLM_ERR_OK is 1
    (src/core/vkllm_errors.inc:6), so a successful run exits with status 1."""
import os
import re
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COMPAT = os.path.join(ROOT, "oracle", "_ref", "compat")
OP_PROGRAMS = ["vkllm_test_op_add", "vkllm_test_op_arg_max", "vkllm_test_op_bin", "vkllm_test_op_copy",
               "vkllm_test_op_embedding", "vkllm_test_op_ffn_up_and_gate", "vkllm_test_op_matmul",
               "vkllm_test_op_permute", "vkllm_test_op_rmsnorm", "vkllm_test_op_rope", "vkllm_test_op_softmax",
               "vkllm_test_op_update_rows", "vkllm_test_tensor_reshape", "vkllm_test_hashmap"]


def program(name):
    path = os.path.join(COMPAT, name)
    if not os.path.exists(path):
        pytest.skip(f"{path} not built (oracle/refpin/Makefile needs the reference checkout)")
    return path


RESHAPE_TABLE_BUGS = {4, 8, 13}  # entries of the reshape program's table with unequal element counts


def failed_cases(out):
    """(test name, loop index) of every "...:<name>:<i>: Failed" line of the check runner."""
    return {(m.group(1), int(m.group(2))) for m in re.finditer(r":(\w+):(\d+): Failed", out)}


def argmax_mismatches_are_ties(out):
    """Every mismatch block the arg_max program prints lists the row with "(gpu max)" and "(host max)"
    marks; True when each block's two marked values are equal."""
    blocks = out.split("Mismatch at index")[1:]
    if not blocks:
        return False
    for b in blocks:
        g = re.search(r"\]: (-?[0-9.]+) \(gpu max\)", b)
        h = re.search(r"\]: (-?[0-9.]+) \(host max\)", b)
        if not g or not h or float(g.group(1)) != float(h.group(1)):
            return False
    return True


@pytest.mark.parametrize("name", OP_PROGRAMS)
def test_reference_op_program_passes(ctx, name):
    r = subprocess.run([program(name)], capture_output=True, text=True, timeout=900)
    out = r.stdout + r.stderr
    summary = [l for l in out.splitlines() if "Checks:" in l]
    assert summary, out[-4000:]
    if "Failures: 0" in summary[-1]:
        assert r.returncode == 0, out[-4000:]
        return
    failed = failed_cases(out)
    if name == "vkllm_test_op_arg_max":
        assert argmax_mismatches_are_ties(out), out[-6000:]
    elif name == "vkllm_test_tensor_reshape":
        assert failed == {("test_tensor_reshape_valid", i) for i in RESHAPE_TABLE_BUGS}, (failed, out[-4000:])
        assert out.count("Assertion 'orig_total == new_total' failed") == len(RESHAPE_TABLE_BUGS), out[-4000:]
    else:
        raise AssertionError(out[-4000:])


def test_reference_token_loop_program(ctx, tiny_gguf, orc):
    import gen_gguf

    path, weights = tiny_gguf
    n_tokens = 40
    r = subprocess.run([program("vkllm_test_infer_gguf"), path, str(n_tokens)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 1, (r.returncode, r.stdout[-2000:], r.stderr[-4000:])  # VKLLM_ERR_OK
    m = re.search(r"input ids: ([0-9 ]+)", r.stderr)
    assert m, r.stderr[-2000:]
    prompt = [int(t) for t in m.group(1).split()]
    names = {"<unk>": 0, "<s>": 1, "</s>": 2}
    toks = [names[t] if t in names else int(t[2:-1]) for t in re.findall(r"<t\d+>|<unk>|<s>|</s>", r.stdout)]
    assert len(toks) == n_tokens, r.stdout[-2000:]
    ref = orc.Llama2(dict(gen_gguf.TINY), weights)
    ref_toks, _ = ref.generate(prompt, n_tokens)
    ref.close()
    assert toks[:32] == ref_toks[:32], (toks, ref_toks)
