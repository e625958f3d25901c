"""CPU: the reference's own engine, speculative-decoding, HTTP API, block and
attention tests, run unmodified with libvllt behind them.

tests/refsuite_plugin.py makes `vllmlite.engine.NumpyRunner` (what
LLMEngine.__init__ constructs, vllmlite/engine.py:46) build a HostRunner over
the host build of libvllt: the backend switch a maintainer would add. The
reference's test files then run as they are, read from the reference's source
tree (this test is skipped where that tree is absent), twice: with the
reference's LLMEngine over that runner (its host sample() on the logits), and
with the product's GpuLLMEngine in LLMEngine's place (device token picks and
run-ahead, as `vllt.engine.gpu_engine` serves):
  * tests/test_engine.py: its invariance grid (block sizes 1-64, prefix
    caching, chunk budgets, no chunking, batch composition, preemption with
    and without the prefix cache), block accounting, prefix-cache hits, stop
    strings, aborts, a prompt larger than the cache, seeded sampling;
  * tests/test_speculative.py: verify, and speculation at k = 1-8 giving the
    same tokens with fewer passes, under preemption, freeing every block;
  * tests/test_api.py: the HTTP server (its engine thread included):
    completions, chat completions, streamed deltas, bad requests, the cache
    metrics and concurrent requests sharing one engine;
  * tests/test_block.py: the block allocator and hash_block's chaining, with
    hash_block itself (and so every prefix-cache lookup of the runs above)
    replaced by the device prefix hash's code compiled for the host;
  * tests/test_attention.py: paged attention against its dense restatement
    (rtol 1e-4) on the reference's grid, with paged_attention replaced by
    vllt.ops.paged_attention, the NumPy-signature drop-in, over the C ABI.
Every one must pass, and the plugin's count shows the passes ran through
libvllt (one runner per engine the tests built).
"""

import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# the reference's source checkout: VLLT_REFERENCE_TREE, else a "reference"
# directory beside this repository
REFERENCE = os.environ.get("VLLT_REFERENCE_TREE", os.path.join(os.path.dirname(ROOT), "reference"))
FILES = ("test_engine.py", "test_speculative.py", "test_api.py", "test_block.py", "test_attention.py")


@pytest.mark.skipif(not all(os.path.exists(os.path.join(REFERENCE, "tests", f)) for f in FILES),
                    reason="the reference's source tree is not here")
@pytest.mark.parametrize("engine", ["reference", "gpu-run-ahead"])
def test_reference_engine_tests_pass_with_libvllt_behind_the_engine(host_library, tmp_path, engine):
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1", VLLT_REFSUITE_BUILD=str(tmp_path),
               VLLT_REFSUITE_LIB=host_library._name, VLLT_REFSUITE_ENGINE=engine,
               PYTHONPATH=os.pathsep.join([os.path.join(ROOT, "tests"), os.path.join(ROOT, "vllm-lite_b200"),
                                           REFERENCE]))
    files = [os.path.join(REFERENCE, "tests", f) for f in FILES]
    # run from a scratch directory: nothing is written into the reference's tree
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "refsuite_plugin", "-p", "no:cacheprovider",
                        *files], cwd=str(tmp_path), env=env, capture_output=True, text=True, timeout=1800)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    m = re.search(r"runners=(\d+) forward_passes=(\d+) block_hashes=(\d+) attention_calls=(\d+)", r.stdout)
    assert m, r.stdout[-2000:]
    runners, passes, hashes, attention = (int(x) for x in m.groups())
    assert runners > 40 and passes > 1000 and hashes > 100 and attention >= 27, r.stdout[-2000:]
    done = re.search(r"(\d+) passed", r.stdout)
    assert done and "failed" not in r.stdout.splitlines()[-1] and int(done.group(1)) >= 90, r.stdout[-2000:]
