// Force-included into the reference's tests/golden_kernel_test.cpp when
// build_ref.sh compiles it for oracle/_ref/ref_packer_pin (test infrastructure):
// its MTRT_GOLDENS_DIR becomes a directory chosen at run time.
#pragma once
const char* pin_goldens_dir();
