python bench.py --no-sub --no-cpu-baseline --steps 20 > gpurun_out/b1.log 2>&1; echo rc=$? >> gpurun_out/b1.log
python bench.py --global-batch 1 --no-sub --no-cpu-baseline --steps 20 > gpurun_out/b_gb1.log 2>&1; echo rc=$? >> gpurun_out/b_gb1.log
for f in b1 b_gb1; do tail -2 gpurun_out/$f.log | python -c "
import sys,json
for l in sys.stdin:
    if l.startswith('{'):
        d=json.loads(l); print('$f', round(d['ms_per_step'],3), round(d['value']/1e6,2), 'e2e', round(d['e2e']['value']/1e6,2))
    else: print(l.strip()[:300])"; done
