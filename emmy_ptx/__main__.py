import sys

from emmy_ptx_b200.compiler import main

sys.exit(main(sys.argv))
