// Status strings and ABI version of the C entry points.
#include "common.cuh"

extern "C" const char* dwarf_status_string(int status) {
  switch (status) {
    case DWARF_OK: return "ok";
    case DWARF_ERR_VERSION: return "ABI version mismatch";
    case DWARF_ERR_NULL: return "required pointer is NULL";
    case DWARF_ERR_SHAPE: return "inconsistent or unsupported shape";
    case DWARF_ERR_STRIDE: return "unsupported stride/layout";
    case DWARF_ERR_ALIGN: return "misaligned pointer or stride";
    case DWARF_ERR_DTYPE: return "unsupported dtype";
    case DWARF_ERR_WORKSPACE: return "workspace missing or too small";
    case DWARF_ERR_LAUNCH: return "CUDA launch failed";
    case DWARF_ERR_VALUE: return "bad scalar argument";
    case DWARF_ERR_SCRATCH_LIMIT: return "problem exceeds the library's built-in scratch size";
    default: return "unknown status";
  }
}

extern "C" int dwarf_abi_version(void) { return DWARF_ABI_VERSION; }
