#!/bin/bash
mkdir -p gpurun_out
rc=0
for m in g d; do
  for v in base poll nopass pollnopass; do echo "=== $v $m"; ./_work/stream_probe_$v $m $([ $v = poll ] && echo 1 || echo 0) || rc=1; done
done
exit $rc
