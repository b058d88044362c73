// Entry point of the oracle/_ref test binary built from the reference's Catch2 sources.
#include <catch2/catch_test_macros.hpp>

int main(int argc, char **argv) { return minicatch::run(argc, argv); }
