"""Generates tests/golden/reference_fixtures.json from the reference's own Zig tests.

Run here, where the reference tree is readable (it is never read at test time):
    python tests/golden/make_golden.py /path/to/peregrine

The reference (Zig + Metal) cannot be built or run on Linux, so its tests are read as
text. The fixtures they hold are extracted:
  * stride golden values: src/model/state.zig:244-254 (fullCacheStrideForMaxSeq);
  * layer topology and dims: src/model/decoder_layer.zig:29-31 (isLinear), block_attn.zig /
    block_linear.zig constants, src/model/dims.zig (hidden row bytes);
  * the persist round-trip byte-pattern fixture: src/server/prefix_persist.zig:457-541
    (token_count, fill order per layer), and the expected-file-bytes test at :443-455;
  * hidden-row byte-pattern cases: src/server/prefix_state_cache.zig:935-1023.
"""
from __future__ import annotations

import json
import re
import sys
from pathlib import Path


def _const(text: str, name: str) -> int:
    """Evaluates a Zig integer constant, resolving other constants it is built from."""
    defs = {m.group(1): m.group(2) for m in re.finditer(
        r"(?:pub )?const (\w+)(?::\s*\w+)?\s*=\s*([0-9A-Za-z_ *+\-()]+);", text)}
    if name not in defs:
        raise SystemExit(f"constant {name} not found")
    expr = defs[name]
    for other in sorted(defs, key=len, reverse=True):
        if other != name and re.search(rf"\b{other}\b", expr):
            expr = re.sub(rf"\b{other}\b", f"({_const(text, other)})", expr)
    return int(eval(expr.replace("_", "") if re.fullmatch(r"[0-9_ *+\-()]+", expr) else expr,
                    {"__builtins__": {}}))


def main(ref: Path) -> dict:
    state = (ref / "src/model/state.zig").read_text()
    stride_cases = []
    for m in re.finditer(r"expectEqual\(@as\(usize, ([0-9_A-Z]+)\), try fullCacheStrideForMaxSeq\(([0-9_A-Z +]+)\)\)", state):
        exp, arg = m.group(1), m.group(2)
        stride_cases.append([arg, exp])
    for m in re.finditer(r"expectError\(error\.InvalidContextLength, fullCacheStrideForMaxSeq\(([0-9_A-Z +]+)\)\)", state):
        stride_cases.append([m.group(1), None])
    max_ctx = 64 * 1024
    assert "MAX_CONTEXT_TOKENS = 64 * 1024" in state

    def ev(s):
        if s is None:
            return None
        s = s.replace("MAX_CONTEXT_TOKENS", str(max_ctx)).replace("_", "")
        return eval(s, {"__builtins__": {}})  # simple integer sums only

    strides = [[ev(a), ev(e)] for a, e in stride_cases]

    attn = (ref / "src/model/block_attn.zig").read_text()
    lin = (ref / "src/model/block_linear.zig").read_text()
    dec = (ref / "src/model/decoder_layer.zig").read_text()
    dims = (ref / "src/model/dims.zig").read_text()
    interval = _const(dec, "FULL_ATTENTION_INTERVAL")
    topology = {
        "num_layers": 32,
        "full_attention_interval": interval,
        "is_linear": [((i + 1) % interval) != 0 for i in range(32)],
        "num_kv": _const(attn, "NUM_KV"),
        "head_dim": _const(attn, "HEAD_DIM"),
        "conv_k": _const(lin, "CONV_K"),
        "conv_dim": _const(lin, "CONV_DIM"),
        "hv": _const(lin, "HV"),
        "dv": _const(lin, "DV"),
        "dk": _const(lin, "DK"),
        "hidden": int(re.search(r"pub const hidden: u32 = (\d+);", dims).group(1)),
    }

    persist = (ref / "src/server/prefix_persist.zig").read_text()
    rt = persist[persist.index('test "save and load round-trip the cached prefix"'):]
    rt = rt[: rt.index("\ntest ")]
    token_count = int(re.search(r"const token_count: usize = (\d+);", rt).group(1))
    cache_init = re.search(r"Cache\.init\((\d+), (\d+)\)", rt)
    fill_start = int(re.search(r"var fill: u8 = (\d+);", rt).group(1))
    efb = persist[persist.index('test "expected file bytes follow the one-model layer topology"'):]
    efb_tokens = int(re.search(r"const token_count: usize = ([0-9_]+);", efb).group(1).replace("_", ""))
    header_fields = re.search(r"const Header = extern struct \{(.*?)\n\};", persist, re.S).group(1)
    header_bytes = 0
    for ty in re.findall(r":\s*(u64|u32),", header_fields):
        size = 8 if ty == "u64" else 4
        header_bytes = (header_bytes + size - 1) // size * size + size
    header_bytes = (header_bytes + 7) // 8 * 8
    magic = int(re.search(r"const MAGIC: u64 = 0x([0-9A-Fa-f_]+);", persist).group(1).replace("_", ""), 16)
    version = int(re.search(r"const VERSION: u32 = (\d+);", persist).group(1))

    psc = (ref / "src/server/prefix_state_cache.zig").read_text()
    hidden_cases = []
    t1 = psc[psc.index('test "storePrefixFromWork marks hidden_valid true for fresh entry'):]
    t1 = t1[: t1.index("\ntest ")]
    hidden_cases.append({
        "name": "fresh entry copies all rows",
        "rows": len(re.search(r"const tokens = \[_\]u32\{ ([0-9, ]+) \}", t1).group(1).split(",")),
        "fill": int(re.search(r"@memset\(work_hidden\.slice\(u8\), 0x([0-9A-F]+)\)", t1).group(1), 16),
    })
    t2 = psc[psc.index('test "storePrefixFromWork preserves reused hidden rows'):]
    t2 = t2[: t2.index("\ntest ")]
    fills = [int(x, 16) for x in re.findall(r"@memset\(hidden_[ab]\.slice\(u8\)(?:\[[^\]]*\])?, 0x([0-9A-F]+)\)", t2)]
    checks = [(int(a) if a else 1, int(b, 16)) for a, b in
              re.findall(r"expectEqual\(@as\(u8, 0x([0-9A-F]+)\), hidden\.slice\(u8\)\[(?:row_bytes \* )?(\d*)\]\)", t2)]
    hidden_cases.append({
        "name": "extend reuses prefix rows and copies suffix rows",
        "prefix_rows": 3, "total_rows": 5, "work_base_row": 3,
        "prefix_fill": fills[0], "suffix_fill": 0x22,
        "checks": [[int(row or 0), val] for val, row in
                   re.findall(r"expectEqual\(@as\(u8, 0x([0-9A-F]+)\), hidden\.slice\(u8\)\[(?:row_bytes \* )?(\d*)\]\)", t2)],
    })
    for c in hidden_cases[1]["checks"]:
        c[1] = int(c[1], 16) if isinstance(c[1], str) else c[1]
    _ = checks

    return {
        "source": "XiaoConstantine/peregrine test blocks, extracted by tests/golden/make_golden.py",
        "stride_cases": strides,
        "topology": topology,
        "persist": {
            "magic": magic, "version": version, "header_bytes": header_bytes,
            "roundtrip_token_count": token_count,
            "roundtrip_cache_init": [int(cache_init.group(1)), int(cache_init.group(2))],
            "fill_start": fill_start,
            "fill_rule": "per layer in order: linear -> conv=fill, recur=fill+1; full -> K=fill, V=fill+1; fill += 2 (u8 wrap)",
            "expected_file_bytes_token_count": efb_tokens,
        },
        "hidden_cases": hidden_cases,
    }


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <path to the peregrine source tree>")
    ref = Path(sys.argv[1])
    out = Path(__file__).resolve().parent / "reference_fixtures.json"
    out.write_text(json.dumps(main(ref), indent=1) + "\n")
    print(out)
