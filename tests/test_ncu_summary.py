"""CPU: the ncu launch-list summariser on a synthetic capture."""
from kernelswift_b200 import ncu_summary as ns

CSV = '''==PROF== Connected to process 1
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","python","h","void ksw::<unnamed>::prep_cast_kernel<float, __nv_bfloat16>(const float *, long)","1","7","(256, 1, 1)","(1, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","500"
"1","1","python","h","void ksw::<unnamed>::moe_grouped_gemm_kernel<0, 1, 256, 0, __nv_bfloat16>(CUtensorMap, CUtensorMap, KParams)","1","7","(320, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","ms","1.5"
"2","1","python","h","void ksw::<unnamed>::sum_topk_kernel<float>(const float *)","1","7","(256, 1, 1)","(4, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","ns","25,000"
"3","1","python","h","void ksw::<unnamed>::moe_grouped_gemm_kernel<0, 1, 256, 0, __nv_bfloat16>(CUtensorMap, CUtensorMap, KParams)","1","7","(320, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","1500"
'''


def test_summary(tmp_path):
    p = tmp_path / "l.csv"
    p.write_text(CSV)
    s = ns.summarize(ns.read_csv(p))
    assert s[0][0].startswith("void moe_grouped_gemm_kernel<0, 1, 256, 0") and s[0][1] == 2
    assert abs(s[0][2] - 3000.0) < 1e-6
    names = [x[0] for x in s]
    assert any("prep_cast" in n for n in names)
    setup = {x[0]: x[3] for x in s}
    assert setup[[n for n in names if "prep_cast" in n][0]] is True
    md = ns.markdown(s, steps=2)
    assert "| 2 | 3000.0 | 1500.0 |" in md and "1.00 | 1500.0 |" in md
    # step share excludes the one-time prep kernel: 3000 / 3025
    assert "99.2%" in md
