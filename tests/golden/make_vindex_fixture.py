"""Copies the reference's smallest on-disk vindex into tests/golden/vindex_ui_walk_trace/.

Run in a container that has the reference tree beside this checkout (or LARQL_REF_ROOT pointing at the
directory that holds larql-main/):

    python tests/golden/make_vindex_fixture.py

Source: crates/larql-python/tests/fixtures/ui_walk_trace_vindex/ of the reference, the fixture its own UI tests
open.  Only the two files the vindex loader reads for the gate walk are copied, byte for byte: index.json
(VindexConfig: 2 layers x 4 features x hidden 8, dtype f32) and gate_vectors.bin (256 bytes of f32 rows).
"""
import os
import shutil

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("LARQL_REF_ROOT", os.path.join(os.path.dirname(ROOT), "reference"))
SRC = os.path.join(REF, "larql-main", "crates", "larql-python", "tests", "fixtures", "ui_walk_trace_vindex")
DST = os.path.join(HERE, "vindex_ui_walk_trace")


def main():
    os.makedirs(DST, exist_ok=True)
    for name in ("index.json", "gate_vectors.bin"):
        shutil.copyfile(os.path.join(SRC, name), os.path.join(DST, name))
        print("copied", name)


if __name__ == "__main__":
    main()
