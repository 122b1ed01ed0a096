"""Regenerate tests/golden/decode_golden.npz from the reference implementation.

Runs the reference project's own fp32 oracle ``paged_attention_decode_reference``
(src/reference.py:8-54, imported from the reference checkout) and its
independent SDPA oracle (tests/oracle_sdpa.py:17-58) on every case of
``golden_cases.py`` and stores, per case, the outputs and a digest of the
inputs. Needs a checkout of the reference project, given as the first
argument or in the ``PAD_REFERENCE_ROOT`` environment variable; the tests
only read the resulting .npz.

    python tests/golden/make_golden.py <path to the reference checkout>
"""

from __future__ import annotations

import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "paged-attention-decode_b200"))
sys.path.insert(0, HERE)
sys.dont_write_bytecode = True

import numpy as np  # noqa: E402
import torch  # noqa: E402

from golden_cases import golden_cases, input_digest  # noqa: E402


def main() -> None:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PAD_REFERENCE_ROOT")
    if not ref_root or not os.path.isfile(os.path.join(ref_root, "src", "reference.py")):
        raise SystemExit("usage: make_golden.py <reference checkout> (or set PAD_REFERENCE_ROOT); "
                         "it must contain src/reference.py")
    sys.path.insert(0, ref_root)
    from src.reference import paged_attention_decode_reference  # the reference's oracle
    from tests.oracle_sdpa import sdpa_oracle  # the reference's independent oracle

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    store = {}
    for name, c in golden_cases():
        args = [torch.from_numpy(np.ascontiguousarray(a)) for a in (c.q, c.k_cache, c.v_cache, c.block_table, c.seq_lens)]
        out = paged_attention_decode_reference(*args).numpy()
        sd = sdpa_oracle(*args, c.page_size).numpy()
        store[f"{name}__out"] = out.astype(np.float32)
        store[f"{name}__sdpa"] = sd.astype(np.float32)
        store[f"{name}__digest"] = np.frombuffer(bytes.fromhex(input_digest(c)), dtype=np.uint8)
        print(f"{name:28s} B={c.q.shape[0]} Hq={c.q.shape[1]} D={c.q.shape[2]} ps={c.page_size} "
              f"max|ref-sdpa|={np.abs(out - sd).max():.2e}")
    path = os.path.join(HERE, "decode_golden.npz")
    np.savez_compressed(path, **store)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
