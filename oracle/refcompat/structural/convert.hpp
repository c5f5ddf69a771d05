// Test infrastructure only.  When oracle/Makefile builds the reference's own
// tests and drivers against this repository's structural:: shim, this
// overlay sits first on the include path so the reference's host converter
// (its tests' CPU truth, any block size) stays the reference's own file,
// named by REF_CONVERT_HPP; every other header comes from the shim.
#pragma once
#include REF_CONVERT_HPP
