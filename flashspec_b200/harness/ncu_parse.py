"""Parse Nsight Compute CSV output and back-fill measured fields of a microbench result.

Restates the behaviour of the reference's scripts/ncu_parse.py (parse the long
``--csv`` format, aggregate bytes and durations over launches, flag kernels that do not
look like the decode kernel) for B200 counters.  Only counter values are read; the
source / SASS pages of a report are never used.
"""

from __future__ import annotations

import csv
import io
from dataclasses import dataclass, field
from typing import Dict, List

# counters the microbench asks ncu for (one pass except the occupancy / stall extras)
FAST_METRICS = (
    "dram__bytes_read.sum",
    "dram__bytes_write.sum",
    "gpu__time_duration.sum",
    "dram__throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__warps_active.avg.pct_of_peak_sustained_active",
    "launch__registers_per_thread",
    "sm__maximum_warps_per_active_cycle_pct",
    "smsp__inst_executed.sum",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
)
STALL_PREFIX = "smsp__average_warps_issue_stalled_"

# kernels whose names mark them as the decode path; anything else captured by the
# filter (e.g. a torch elementwise kernel) is flagged as suspicious
DECODE_KERNEL_HINTS = ("decode_kernel", "merge_partials_kernel", "page_update_kernel", "quantize_blocks_kernel")

_UNIT_SCALE = {
    "byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "KB": 1e3, "MB": 1e6, "GB": 1e9,
    "nsecond": 1.0, "usecond": 1e3, "msecond": 1e6, "second": 1e9, "ns": 1.0, "us": 1e3, "ms": 1e6,
}


@dataclass
class KernelMetrics:
    name: str
    launches: int = 0
    metrics: Dict[str, List[float]] = field(default_factory=dict)

    def total(self, key: str) -> float:
        return float(sum(self.metrics.get(key, [])))

    def mean(self, key: str) -> float:
        v = self.metrics.get(key, [])
        return float(sum(v) / len(v)) if v else 0.0


def _to_float(value: str, unit: str) -> float:
    v = float(value.replace(",", ""))
    return v * _UNIT_SCALE.get(unit, 1.0)


def parse_ncu_csv(text: str) -> Dict[str, KernelMetrics]:
    """Parse ``ncu --csv`` (long format: one row per launch x metric).  Lines before the
    header (``==PROF==`` banners, program output) are skipped.  Bytes are normalised to
    bytes and durations to nanoseconds."""
    lines = text.splitlines()
    start = next((i for i, l in enumerate(lines) if l.startswith('"ID"') or l.startswith("ID,")), None)
    if start is None:
        raise ValueError("no ncu CSV header found")
    rows = list(csv.reader(io.StringIO("\n".join(lines[start:]))))
    hdr = rows[0]
    try:
        i_id, i_name = hdr.index("ID"), hdr.index("Kernel Name")
        i_metric, i_value = hdr.index("Metric Name"), hdr.index("Metric Value")
    except ValueError as exc:
        raise ValueError(f"unexpected ncu CSV header: {hdr}") from exc
    i_unit = hdr.index("Metric Unit") if "Metric Unit" in hdr else None
    out: Dict[str, KernelMetrics] = {}
    seen = set()
    for r in rows[1:]:
        if len(r) <= max(i_id, i_name, i_metric, i_value):
            continue
        name = r[i_name]
        k = out.setdefault(name, KernelMetrics(name))
        if (r[i_id], name) not in seen:
            seen.add((r[i_id], name))
            k.launches += 1
        try:
            v = _to_float(r[i_value], r[i_unit] if i_unit is not None else "")
        except ValueError:
            continue
        k.metrics.setdefault(r[i_metric], []).append(v)
    return out


def suspicious_kernels(parsed: Dict[str, KernelMetrics]) -> List[str]:
    return [n for n in parsed if not any(h in n for h in DECODE_KERNEL_HINTS)]


def apply_backfill(result: dict, parsed: Dict[str, KernelMetrics]) -> List[str]:
    """Fill the ``measured_*`` fields of a microbench result from parsed ncu output
    (sums over launches for bytes/time, duration-weighted means for percentages, the
    dominant kernel's registers and occupancy ceiling).  Returns the suspicious
    kernel names and records a ``profiler_warning`` when there are any."""
    bad = suspicious_kernels(parsed)
    if not parsed:
        return bad
    dram = sum(k.total("dram__bytes_read.sum") + k.total("dram__bytes_write.sum") for k in parsed.values())
    dur = sum(k.total("gpu__time_duration.sum") for k in parsed.values())
    launches = sum(k.launches for k in parsed.values())
    dominant = max(parsed.values(), key=lambda k: k.total("gpu__time_duration.sum"))

    def weighted(key):
        num = sum(k.total("gpu__time_duration.sum") * k.mean(key) for k in parsed.values() if key in k.metrics)
        return num / dur if dur > 0 else None

    result["measured_dram_bytes"] = dram
    result["measured_ncu_kernel_duration_ms"] = dur / 1e6
    result["measured_ncu_kernel_count"] = launches
    result["measured_ncu_kernel_names"] = sorted(parsed)
    result["measured_achieved_bandwidth_gbps"] = dram / dur if dur > 0 else None  # bytes/ns == GB/s
    result["measured_dram_throughput_pct"] = weighted("dram__throughput.avg.pct_of_peak_sustained_elapsed")
    result["measured_sm_utilization_pct"] = weighted("sm__throughput.avg.pct_of_peak_sustained_elapsed")
    result["measured_occupancy_pct"] = weighted("sm__warps_active.avg.pct_of_peak_sustained_active")
    result["measured_tensor_pipe_pct"] = weighted("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active")
    result["measured_registers_per_thread"] = dominant.mean("launch__registers_per_thread") or None
    result["measured_theoretical_occupancy_pct"] = dominant.mean("sm__maximum_warps_per_active_cycle_pct") or None
    result["measured_inst_executed"] = sum(k.total("smsp__inst_executed.sum") for k in parsed.values()) or None
    stalls = {m[len(STALL_PREFIX):]: dominant.mean(m) for m in dominant.metrics if m.startswith(STALL_PREFIX)}
    if stalls:
        result["measured_stall_breakdown"] = stalls
    result["bandwidth_fields_are_estimates"] = False
    if bad:
        result["profiler_warning"] = f"non-decode kernels captured: {bad}"
    return bad
