// plugin/plugin-context.h -- IN-REPO STUB of vpipe's plugin context.
//
// The reference's registration (src/ltx25-plugin.cc:70-134) calls six
// extension points on vpipe::VpipePluginContext: register_video_family,
// register_stage, register_vae_family, register_quantize_family,
// register_metal_library and register_catalog_entries.  The B200 plugin
// shim replaces only the kernel half of that: where the reference hands the
// host three metallibs "under the names the model layer resolves with
// load_library()" (src/ltx25-plugin.cc:117-133), the shim hands it one
// named CUDA kernel table.  This stub declares that seam, plus the lookup
// the model layer does, and nothing else; the family, stage, VAE,
// quantize-family and catalog registrations stay the reference plugin's own
// code and need the real SDK.
#pragma once

#include <cstddef>

namespace vpipe {

// One registered kernel library: a name, the backend it runs on, and the
// table of entry points (a C struct whose first int is its own version, so
// a model layer built against another version refuses it by name).
struct KernelTable {
  const char* name;
  const char* backend;
  const void* table;
  std::size_t table_bytes;
};

class VpipePluginContext {
public:
  virtual ~VpipePluginContext() = default;

  // The counterpart of register_metal_library(name, bytes, len): the
  // kernels before anything can dispatch them.  First registration of a
  // name wins; a later one with the same name is refused (false).
  virtual bool register_kernel_table(const KernelTable& t) = 0;

  // What the model layer calls to resolve a library by name (the
  // reference's load_library()); null when nothing registered it.
  virtual const KernelTable* find_kernel_table(const char* name) const = 0;
};

}  // namespace vpipe
