"""Regenerate tests/golden/yolo_proto_fields.json from the reference's proto/yolo.proto.

The serving layer builds the proto's message types from descriptors at run time (protoc is
not available); this fixture pins every message's fields (name, number, type, repeated)
and the service's methods, read from the reference's own .proto text, so a test can check
that the run-time descriptors are wire-compatible with the reference's clients.

    python tests/golden/make_proto_fields.py --ref <reference checkout>
"""
from __future__ import annotations

import argparse
import json
import os
import re


def parse(text: str) -> dict:
    text = re.sub(r"//[^\n]*", "", text)
    out = {"package": re.search(r"\bpackage\s+([\w.]+)\s*;", text).group(1),
           "messages": {}, "services": {}}
    for name, body in re.findall(r"\bmessage\s+(\w+)\s*\{([^}]*)\}", text):
        fields = []
        for rep, ftype, fname, num in re.findall(
                r"(repeated\s+)?([\w.]+)\s+(\w+)\s*=\s*(\d+)\s*;", body):
            fields.append({"name": fname, "number": int(num), "type": ftype,
                           "repeated": bool(rep)})
        out["messages"][name] = fields
    for name, body in re.findall(r"\bservice\s+(\w+)\s*\{([^}]*)\}", text):
        out["services"][name] = [
            {"name": m, "input": i, "output": o}
            for m, i, o in re.findall(r"rpc\s+(\w+)\s*\(\s*(\w+)\s*\)\s*returns\s*\(\s*(\w+)\s*\)",
                                      body)]
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference checkout (holds proto/yolo.proto)")
    a = ap.parse_args()
    with open(os.path.join(a.ref, "proto", "yolo.proto")) as f:
        spec = parse(f.read())
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "yolo_proto_fields.json")
    with open(dst, "w") as f:
        json.dump(spec, f, indent=1, sort_keys=True)
    print("wrote", dst)


if __name__ == "__main__":
    main()
