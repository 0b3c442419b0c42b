"""Test helper: serves the reference gateway's functions (oracle/_ref/libkib_ref.so,
ref_gw_* from oracle/ref_gateway_shim.cpp) over stdin/stdout, one JSON request per
line.  A separate process because the reference library's iostream code cannot run
in a process that has already loaded numpy or torch (their C++ runtime comes
first); this one imports neither."""
import base64
import ctypes
import json
import sys


def main(path):
    lib = ctypes.CDLL(path)
    P, U, I, L = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int64
    fns = {}
    for name, args in (("describe", [I, ctypes.c_char_p, U, P, U]), ("split_reasoning", [ctypes.c_char_p, U, I, I, P, U]),
                       ("stream_reasoning", [ctypes.c_char_p, P, U, I, I, P, U]), ("body", [I, P, P, P, U])):
        f = getattr(lib, "ref_gw_" + name)
        f.argtypes, f.restype = args, L
        fns[name] = f

    def call(f):
        n = f(None, 0)
        buf = ctypes.create_string_buffer(max(1, n))
        f(buf, n)
        return buf.raw[:n]

    for line in sys.stdin:
        q = json.loads(line)
        fn = q["fn"]
        if fn == "describe":
            b = base64.b64decode(q["body"])
            r = call(lambda o, n: fns["describe"](q["kind"], b, len(b), o, n))
        elif fn == "split_reasoning":
            t = base64.b64decode(q["text"])
            r = call(lambda o, n: fns["split_reasoning"](t, len(t), q["think"], q["fmt"], o, n))
        elif fn == "stream_reasoning":
            pieces = [base64.b64decode(p) for p in q["pieces"]]
            j = b"".join(pieces)
            lens = (ctypes.c_uint64 * max(1, len(pieces)))(*[len(p) for p in pieces])
            r = call(lambda o, n: fns["stream_reasoning"](j, lens, len(pieces), q["think"], q["fmt"], o, n))
        else:
            s = (ctypes.c_char_p * 8)(*[x.encode() for x in q["strs"]], *([None] * (8 - len(q["strs"]))))
            v = (ctypes.c_int64 * 8)(*q["nums"], *([0] * (8 - len(q["nums"]))))
            r = call(lambda o, n: fns["body"](q["which"], s, v, o, n))
        sys.stdout.write(base64.b64encode(r).decode() + "\n")
        sys.stdout.flush()


if __name__ == "__main__":
    main(sys.argv[1])
