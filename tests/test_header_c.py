"""include/hla_s6.h is a plain C header: a C11 translation unit that includes it, calls entry points
through their declared prototypes and links against libhla_s6.so builds with gcc and runs on a host
without a GPU (argument validation returns the documented status codes before any device work).
This is how a non-Python host (a cgo / JNI / C++ binding) consumes the boundary.  CPU only."""
import shutil
import subprocess
import tempfile
from pathlib import Path

import pytest

from conftest import ROOT, pkg

C_SOURCE = r'''
#include <stdio.h>
#include <string.h>
#include "hla_s6.h"

int main(void) {
  if (hla_s6_version() != HLA_S6_ABI_VERSION) return 10;
  /* page 5 is refused on the host, before any CUDA call */
  int rc = hla_s6_history_attention(0, 0, 0, 0, 1, 0, 0, 0, 0, 0, 0, 0, 1, 16, 512, 5, 1.0f, 1, 0, 0, 0, 0, 0, 0,
                                    0, 0);
  if (rc != HLA_S6_EINVAL || !strstr(hla_s6_last_error(), "page")) return 11;
  /* unknown flags of the split stage */
  rc = hla_s6_history_partials(0, 0, 0, 0, 1, 0, 0, 0, 0, 0, 0, 1, 16, 512, 16, 1.0f, 1, 0, 0, 0, 0x40, 0);
  if (rc != HLA_S6_EINVAL || !strstr(hla_s6_last_error(), "flags")) return 12;
  /* the fixed-scratch entry refuses a call beyond its array */
  rc = hla_s6_history_attention_static(0, 0, 0, 0, 1, 0, 0, 0, 0, 0, 0, 0, 64, 16, 512, 16, 1.0f, 16, 0, 0, 0, 0, 0,
                                       0);
  if (rc != HLA_S6_EOVERFLOW) return 13;
  /* bounded waits: process-wide limit, 0 restores the 2 s default */
  if (hla_s6_set_wait_limit_ns(1000000ull) != 2000000000ull) return 14;
  if (hla_s6_set_wait_limit_ns(0) != 1000000ull) return 15;
  printf("ok %d\n", hla_s6_version());
  return 0;
}
'''


@pytest.mark.skipif(shutil.which('gcc') is None, reason='gcc not installed')
def test_c_host_compiles_links_and_gets_status_codes():
    lib = Path(pkg('build').build())
    with tempfile.TemporaryDirectory() as d:
        src, exe = Path(d) / 'host.c', Path(d) / 'host'
        src.write_text(C_SOURCE)
        cc = subprocess.run(['gcc', '-std=c11', '-Wall', '-Werror', '-I', str(ROOT / 'include'), str(src), '-o',
                             str(exe), '-L', str(lib.parent), '-lhla_s6', f'-Wl,-rpath,{lib.parent}'],
                            capture_output=True, text=True)
        assert cc.returncode == 0, cc.stderr
        run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
        assert run.returncode == 0, (run.returncode, run.stdout, run.stderr)
        assert run.stdout.strip() == f'ok {pkg("_lib").ABI_VERSION}'
