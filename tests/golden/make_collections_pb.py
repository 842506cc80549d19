"""Writes the protobuf state-dictionary fixtures with Google's protobuf runtime (an encoder independent of
common_b200.collections_pb), from the message definitions of engine/ml/src/main/proto/collections.proto
restated as descriptors below.

  collections_small.pb     packed encoding (proto3 default), as the reference's StateDictionary.save writes
  collections_unpacked.pb  the same messages with every repeated scalar unpacked (a form parsers must accept)
  collections_expected.npz the values each key must decode to (CollectionEncoder.decode semantics)

Run from the repository root:  python tests/golden/make_collections_pb.py
"""
import os

import numpy as np
from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

HERE = os.path.dirname(os.path.abspath(__file__))

F = descriptor_pb2.FieldDescriptorProto


def build_classes(packed: bool, name: str):
    fd = descriptor_pb2.FileDescriptorProto(name=name, package="fixture_" + name.split(".")[0], syntax="proto3")

    def msg(mname, fields):
        m = fd.message_type.add(name=mname)
        for fname, num, ftype, label, tname in fields:
            f = m.field.add(name=fname, number=num, type=ftype, label=label)
            if tname:
                f.type_name = tname
            if label == F.LABEL_REPEATED and ftype != F.TYPE_MESSAGE and not packed:
                f.options.packed = False

    pkg = "." + fd.package + "."
    msg("TraversalPolicyData", [("dims", 1, F.TYPE_INT32, F.LABEL_REPEATED, None),
                                ("traversal_axis", 2, F.TYPE_INT32, F.LABEL_OPTIONAL, None)])
    msg("CollectionData", [("traversal_policy", 1, F.TYPE_MESSAGE, F.LABEL_OPTIONAL, pkg + "TraversalPolicyData"),
                           ("data", 2, F.TYPE_DOUBLE, F.LABEL_REPEATED, None),
                           ("data_32", 3, F.TYPE_FLOAT, F.LABEL_REPEATED, None)])
    msg("CollectionLibraryEntry", [("key", 1, F.TYPE_STRING, F.LABEL_OPTIONAL, None),
                                   ("collection", 2, F.TYPE_MESSAGE, F.LABEL_OPTIONAL, pkg + "CollectionData")])
    msg("CollectionLibraryData", [("collections", 1, F.TYPE_MESSAGE, F.LABEL_REPEATED,
                                   pkg + "CollectionLibraryEntry")])
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fd)
    return {n: message_factory.GetMessageClass(pool.FindMessageTypeByName(fd.package + "." + n))
            for n in ("TraversalPolicyData", "CollectionData", "CollectionLibraryEntry", "CollectionLibraryData")}


def library(cls, cases):
    lib = cls["CollectionLibraryData"]()
    for key, dims, axis, data, data32 in cases:
        e = lib.collections.add()
        e.key = key
        if dims is not None:
            e.collection.traversal_policy.dims.extend(dims)
            e.collection.traversal_policy.traversal_axis = axis
        e.collection.data.extend(data)
        e.collection.data_32.extend(data32)
    return lib


def cases():
    rng = np.random.default_rng(7)
    a = rng.standard_normal((2, 3)).astype(np.float32)
    b = rng.standard_normal(4)
    c3 = rng.standard_normal((2, 2, 3)).astype(np.float32)
    both64 = rng.standard_normal(3)
    both32 = rng.standard_normal(3).astype(np.float32)
    return [
        # key, dims, traversal_axis, data (f64), data_32 (f32)
        ("model.a_f32", [2, 3], 0, [], a.ravel().tolist()),
        ("model.b_f64", [4], 1, b.tolist(), []),
        ("model.c_3d", [2, 2, 3], 2, [], c3.ravel().tolist()),
        ("model.null", None, 0, [], []),                    # no dimensions: decodes to null, dropped
        ("model.both", [3], 0, both64.tolist(), both32.tolist()),  # `data` wins over `data_32`
        ("model.a_f32", [2, 3], 0, [], (a.ravel() * 2).tolist()),  # a later entry replaces an earlier key
        ("model.empty_f32", [0], 0, [], []),               # a zero-length dimension, no values
    ], {
        "model.a_f32": a * 2, "model.b_f64": b, "model.c_3d": c3, "model.both": both64,
        "model.empty_f32": np.zeros(0, np.float32),
    }


def main():
    cs, expected = cases()
    for packed, fname in ((True, "collections_small.pb"), (False, "collections_unpacked.pb")):
        cls = build_classes(packed, fname.replace(".pb", ".proto"))
        with open(os.path.join(HERE, fname), "wb") as f:
            f.write(library(cls, cs).SerializeToString())
    np.savez(os.path.join(HERE, "collections_expected.npz"), **{k.replace(".", "__"): v for k, v in expected.items()})


if __name__ == "__main__":
    main()
