"""Summarise `ncu --csv --page raw` exports as a markdown table.

    python -m flashattn_cuda.ncu_extract --prefill p.csv --decode d.csv --out summary.md

Same job as the reference's bench/ncu_extract.py (kernel-name shortening,
raw-CSV parsing, a per-kernel table with unit normalisation), with the
figures that bound these kernels on B200: tensor-pipe and MUFU utilisation
for prefill, DRAM bytes and throughput for decode. Runs without a GPU.
"""

import argparse
import csv
import os
import re

# (metric, label, format) in table order.
METRICS = [
    ("gpu__time_duration.sum", "Kernel duration", "{:,.0f} ns"),
    ("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
     "Tensor pipe active", "{:.1f}%"),
    ("sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active",
     "MUFU (XU) pipe", "{:.1f}%"),
    ("smsp__issue_active.avg.pct_of_peak_sustained_active", "Issue slots busy",
     "{:.1f}%"),
    ("sm__warps_active.avg.pct_of_peak_sustained_active", "Achieved occupancy",
     "{:.1f}%"),
    ("gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
     "DRAM throughput", "{:.1f}%"),
    ("dram__bytes_read.sum.per_second", "DRAM read bandwidth", "{:.1f} GB/s"),
    ("dram__bytes_read.sum", "DRAM bytes read", "{:,.0f} B"),
    ("dram__bytes_write.sum", "DRAM bytes written", "{:,.0f} B"),
    ("launch__registers_per_thread", "Registers / thread", "{:.0f}"),
]

# ncu picks a unit per value; normalise throughput to GB/s and sizes to bytes.
RATE_TO_GBS = {"byte/second": 1e-9, "Kbyte/second": 1e-6, "Mbyte/second": 1e-3,
               "Gbyte/second": 1.0, "Tbyte/second": 1e3, "byte/s": 1e-9,
               "Kbyte/s": 1e-6, "Mbyte/s": 1e-3, "Gbyte/s": 1.0, "Tbyte/s": 1e3}
SIZE_TO_B = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
TIME_TO_NS = {"nsecond": 1.0, "usecond": 1e3, "msecond": 1e6, "second": 1e9,
              "ns": 1.0, "us": 1e3, "ms": 1e6, "s": 1e9}


def short_kernel_name(name):
    """Drops the return type, namespaces and parameter list of a demangled
    kernel name but keeps template arguments, so instantiations stay
    distinguishable: 'void fa::prefill::prefill_kernel<(bool)1>(int)' ->
    'prefill_kernel<(bool)1>'."""
    s = name.strip()
    # cut the parameter list: the first '(' at template depth 0 that is not
    # part of "(anonymous namespace)" or a "(bool)" style template argument
    depth, cut = 0, len(s)
    i = 0
    while i < len(s):
        c = s[i]
        if c == "<":
            depth += 1
        elif c == ">":
            depth -= 1
        elif c == "(" and depth == 0:
            if s.startswith("(anonymous namespace)", i):
                i += len("(anonymous namespace)")
                continue
            cut = i
            break
        i += 1
    s = s[:cut].strip()
    if s.startswith("void "):
        s = s[5:]
    # remove qualifiers outside template arguments
    depth, last = 0, -1
    for i, c in enumerate(s):
        if c == "<":
            depth += 1
        elif c == ">":
            depth -= 1
        elif c == ":" and depth == 0 and i + 1 < len(s) and s[i + 1] == ":":
            last = i + 1
    return s[last + 1:] if last >= 0 else s


def _number(text):
    text = text.replace(",", "").strip()
    try:
        return float(text)
    except ValueError:
        return None


def parse(path):
    """{kernel: {metric: (value, unit)}} from an ncu raw CSV (first launch of
    each kernel name)."""
    if not os.path.exists(path):
        raise SystemExit(f"missing ncu export: {path}")
    with open(path, newline="", encoding="utf-8") as fh:
        rows = list(csv.reader(fh))
    # long format (--print-... with "Metric Name" / "Metric Value" columns)
    for i, row in enumerate(rows):
        if "Metric Name" in row and "Metric Value" in row:
            col = {n: j for j, n in enumerate(row)}
            kcol = col.get("Kernel Name", col.get("Function Name"))
            if kcol is None:
                raise SystemExit(f"{path}: no kernel-name column")
            out = {}
            for r in rows[i + 1:]:
                if len(r) <= col["Metric Value"]:
                    continue
                v = _number(r[col["Metric Value"]])
                if v is None:
                    continue
                unit = r[col["Metric Unit"]] if "Metric Unit" in col else ""
                out.setdefault(r[kcol], {}).setdefault(r[col["Metric Name"]], (v, unit))
            if not out:
                raise SystemExit(f"{path}: no metric rows")
            return out
    # wide format of `--page raw --csv`: header row of metric names, a units
    # row, then one row per launch
    for i, row in enumerate(rows):
        if "Kernel Name" in row and i + 2 < len(rows) + 1:
            kcol = row.index("Kernel Name")
            units = rows[i + 1] if i + 1 < len(rows) else []
            out = {}
            for r in rows[i + 2:]:
                if len(r) != len(row):
                    continue
                d = out.setdefault(r[kcol], {})
                for j, name in enumerate(row):
                    v = _number(r[j])
                    if v is not None and name not in d:
                        d[name] = (v, units[j] if j < len(units) else "")
            if out:
                return out
    raise SystemExit(f"{path}: no CSV header with metric columns")


def _normalise(metric, value, unit):
    if metric.endswith("per_second"):
        return value * RATE_TO_GBS.get(unit, 1.0)
    if unit in SIZE_TO_B:
        return value * SIZE_TO_B[unit]
    if unit in TIME_TO_NS:
        return value * TIME_TO_NS[unit]
    return value


def kernel_table(parsed):
    """Markdown table, one column per kernel; metrics absent from every
    kernel are left out rather than shown as zero."""
    kernels = list(parsed)
    names = [short_kernel_name(k) for k in kernels]
    lines = ["| metric | " + " | ".join(f"`{n}`" for n in names) + " |",
             "|---|" + "---|" * len(kernels)]
    for metric, label, fmt in METRICS:
        cells, any_value = [], False
        for k in kernels:
            if metric in parsed[k]:
                v, unit = parsed[k][metric]
                cells.append(fmt.format(_normalise(metric, v, unit)))
                any_value = True
            else:
                cells.append("n/a")
        if any_value:
            lines.append(f"| {label} | " + " | ".join(cells) + " |")
    return "\n".join(lines) + "\n"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--prefill")
    ap.add_argument("--decode")
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    parts = ["# ncu summary\n"]
    for label, path in (("prefill", a.prefill), ("decode", a.decode)):
        if path:
            parts.append(f"\n## {label}\n\n" + kernel_table(parse(path)))
    with open(a.out, "w", encoding="utf-8") as fh:
        fh.write("".join(parts))


if __name__ == "__main__":
    main()
