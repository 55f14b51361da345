"""Generate tests/golden/*.npz from the reference's own ATen implementation.

The reference (FlashEngine.cpp src/portable_gpu_ops.cpp) is compiled for the
CPU by oracle/build_oracle.py into oracle/_ref/libfe_ref_aten.so; this script
runs its ``store`` (append) and ``prepare_plan`` + ``attention`` on every case
of tests/golden/cases.py and stores:

  meta_*         the step metadata (qo, kv, pages, last, slots)
  input_sha256   digest of the seeded inputs (see cases.input_digest)
  inputs (small cases only): kpool, vpool, knew, vnew, q
  ref_out        the reference attention output (uint16 bit patterns)
  ref_k_rows, ref_v_rows  pool rows at every written slot after the reference store
  ref_k_sha256, ref_v_sha256  digests of the full pools after the reference store

Run in a container that has the reference tree:
``python tests/golden/make_golden.py``.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402

ROOT = cases.ROOT
sys.path.insert(0, ROOT)
import oracle  # noqa: E402


def run_reference(case):
    inp = case.inputs()
    md = case.metadata()
    ref = oracle.RefAten(case.hq, case.hkv, case.dim, case.page, md.batch, case.max_pages(),
                         case.bf16, case.num_blocks)
    kpool, vpool = inp["kpool"].copy(), inp["vpool"].copy()
    ref.store(inp["knew"], inp["vnew"], kpool, vpool, md.slots)
    ref.prepare(md.qo, md.kv, md.pages, md.last)
    out = ref.attention(inp["q"], kpool, vpool, case.causal)
    ref.close()
    return inp, md, kpool, vpool, out


def main():
    oracle.build_oracle.build_reference()
    for case in cases.all_cases():
        inp, md, kpool, vpool, out = run_reference(case)
        written = np.where(md.slots >= 0, md.slots, case.cache_slots - 1)
        data = {
            "meta_qo": md.qo, "meta_kv": md.kv, "meta_pages": md.pages, "meta_last": md.last,
            "meta_slots": md.slots,
            "input_sha256": np.array(cases.input_digest(inp)),
            "ref_out": out,
            "ref_k_rows": kpool[written], "ref_v_rows": vpool[written],
            "ref_k_sha256": np.array(hashlib.sha256(kpool.tobytes()).hexdigest()),
            "ref_v_sha256": np.array(hashlib.sha256(vpool.tobytes()).hexdigest()),
        }
        if case.store_inputs:
            data.update(inp)
        np.savez_compressed(cases.fixture_path(case.name), **data)
        size = os.path.getsize(cases.fixture_path(case.name))
        print(f"{case.name}: rows={md.rows} batch={md.batch} -> {size/1024:.1f} KiB")


if __name__ == "__main__":
    main()
