#!/bin/sh
# Prints the options GCC's -march=native expands to on the host that runs
# this script (the -m..., -mtune=... and --param ... cache sizes), on one
# line.  oracle/native_march.txt holds this line as printed on the B200
# bench host; oracle/Makefile builds the reference with it (target
# ref-native), which is the reference's own -march=native build for that
# host (CMakeLists.txt:14), made from the sources where they lie.
${CC:-gcc} -march=native -E -v - </dev/null 2>&1 | grep '/cc1 ' | head -1 |
  tr ' ' '\n' |
  awk 'p == 1 { printf " --param %s", $0; p = 0; next }
       $0 == "--param" { p = 1; next }
       /^-march=|^-mtune=|^-m[a-z0-9]/ { printf " %s", $0 }
       END { printf "\n" }' | sed 's/^ //'
