// Catch2 runner for the reference's own verifier tests (tests/test_speculative_verifier.cpp),
// compiled from the reference tree by oracle/Makefile into oracle/_ref/. Test infrastructure only.
#define CATCH_CONFIG_MAIN
#include "catch.hpp"
