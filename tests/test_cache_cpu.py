"""Host side of the on-disk weight cache: the fingerprint prefix is the worker's (FNV-1a 32 over
UTF-16 code units, worker.js:31, 100) and pruning keeps only the current prefix (worker.js:82-88)."""
import os

from conftest import load_package


def _js_fnv(s):
    """worker.js:31 as written: for (const c of s) iterates code points, c.charCodeAt(0) is the first
    UTF-16 unit of each; Math.imul keeps the low 32 bits."""
    h = 0x811C9DC5
    for ch in s:
        unit = ord(ch) if ord(ch) < 0x10000 else 0xD800 + ((ord(ch) - 0x10000) >> 10)
        h = ((h ^ unit) * 0x01000193) & 0xFFFFFFFF
    return f"{h:08x}"


def test_fnv_known_values():
    pkg = load_package()
    assert pkg.fnv1a32("") == "811c9dc5"
    assert pkg.fnv1a32("a") == "e40c292c"          # FNV-1a 32 test vector
    assert pkg.fnv1a32("foobar") == "bf9cf968"     # FNV-1a 32 test vector


def test_fnv_matches_worker_loop():
    pkg = load_package()
    for s in ("https://cdn.example/assets/", '{"layer_types": ["linear_attention"]}', "héllo wörld", "emoji \U0001F600!"):
        assert pkg.fnv1a32(s) == _js_fnv(s)


def test_prefix_and_prune(tmp_path):
    pkg = load_package()
    pre = pkg.cache_prefix("v19-test", "https://a/", "{}", '{"shards": []}')
    assert pre.startswith("v19-test__") and pre.endswith("__") and len(pre) == len("v19-test__") + 8 + 2
    old = pkg.cache_prefix("v19-test", "https://a/", "{}", '{"shards": [1]}')
    assert old != pre
    cache = pkg.WeightCache(str(tmp_path), pre)
    for name in (pre + "a.s4w", old + "a.s4w", old + "b.s4w", "other.txt"):
        (tmp_path / name).write_bytes(b"x")
    assert cache.prune() == 2
    assert sorted(os.listdir(tmp_path)) == sorted([pre + "a.s4w", "other.txt"])
    assert cache.path("layers.0/mlp.q") == os.path.join(str(tmp_path), pre + "layers.0_mlp.q.s4w")


def _header(N, K, flags=0, wq=None, ws=None, wb=None, magic=0x4C573453, version=1):
    import struct
    nblk, kt = (N + 127) // 128, (K + 63) // 64
    wq = nblk * kt * 4096 if wq is None else wq
    ws = nblk * kt * 512 if ws is None else ws
    wb = (ws if flags & 1 else 0) if wb is None else wb
    return struct.pack("<IIiiIIQQQQQ", magic, version, N, K, flags, 0, wq, ws, wb, 0, 0)


def test_load_rejects_bad_entries_before_allocating(tmp_path):
    """s4_weight_load checks the header and the file length before sizing any buffer from the
    header: a damaged entry whose header claims a 64 GB payload, a foreign file, inconsistent
    sections or a short payload are S4_ERR_IO without host or device allocation. The validation
    never dereferences the context, so a zeroed stand-in suffices here (no GPU)."""
    import ctypes
    pkg = load_package()
    lib = pkg.load_library()
    fake_ctx = ctypes.create_string_buffer(4096)
    cases = {
        "huge": _header(128, 1 << 30),                       # consistent sections, 64 GB claimed
        "magic": _header(128, 2048, magic=0x12345678) + bytes(4608 * 32),
        "flags": _header(128, 2048, flags=4) + bytes(4608 * 32),
        "sections": _header(128, 2048, wq=4096) + bytes(4608 * 32),
        "short": _header(128, 2048) + bytes(4608 * 32 - 1),
        "long": _header(128, 2048) + bytes(4608 * 32 + 16),
        "shape": _header(0, 2048),
    }
    for name, data in cases.items():
        p = tmp_path / f"{name}.s4w"
        p.write_bytes(data)
        out = ctypes.c_void_p()
        rc = lib.s4_weight_load(ctypes.addressof(fake_ctx), str(p).encode(), ctypes.byref(out))
        assert rc == pkg.s4mm.ERR_IO, (name, rc, lib.s4_last_error())
        assert not out.value, name


def _checksum(p, h=0xCBF29CE484222325):
    """The cache payload checksum (FNV-1a style over little-endian 8-byte words, xor-shift per word)."""
    m = (1 << 64) - 1
    n, i = len(p), 0
    while i + 8 <= n:
        h = ((h ^ int.from_bytes(p[i:i + 8], "little")) * 0x100000001B3) & m
        h ^= h >> 29
        i += 8
    w = int.from_bytes(p[i:] + bytes(8 - (n - i)), "little")
    h = ((h ^ w ^ n) * 0x100000001B3) & m
    return h ^ (h >> 29)


def test_load_accepts_a_valid_entry_up_to_the_device(tmp_path):
    """A well-formed entry passes every file check and stops only at the device upload (no GPU
    here: S4_ERR_CUDA); the same entry with one payload byte flipped is S4_ERR_IO (checksum)."""
    import ctypes
    import struct
    pkg = load_package()
    lib = pkg.load_library()
    fake_ctx = ctypes.create_string_buffer(4096)
    payload = bytes((i * 37) & 0xFF for i in range(4608 * 32))
    good = bytearray(_header(128, 2048) + payload)
    struct.pack_into("<Q", good, 48, _checksum(payload))
    bad = bytearray(good)
    bad[64 + 1000] ^= 1
    for name, data, want in (("good", good, pkg.s4mm.ERR_CUDA), ("flipped", bad, pkg.s4mm.ERR_IO)):
        p = tmp_path / f"{name}.s4w"
        p.write_bytes(bytes(data))
        out = ctypes.c_void_p()
        rc = lib.s4_weight_load(ctypes.addressof(fake_ctx), str(p).encode(), ctypes.byref(out))
        assert rc == want, (name, rc, lib.s4_last_error())
        assert not out.value, name
