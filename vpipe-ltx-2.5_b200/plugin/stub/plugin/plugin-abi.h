// plugin/plugin-abi.h -- IN-REPO STUB of the vpipe plugin ABI header.
//
// The vpipe SDK is not part of this repository.  The reference plugin
// (src/ltx25-plugin.cc) includes "plugin/plugin-abi.h" for the plugin info
// record, the host-feature names it requires and VPIPE_PLUGIN_DEFINE; this
// stub declares exactly those, with the shapes the reference uses them in
// (plugin ABI 8, README.md "Building"), so the B200 plugin shim compiles and
// can be loaded by a test host without vpipe.  Against a real vpipe install
// the SDK's own header replaces this one on the include path.
//
// The exported symbol names below are this stub's; the SDK's own are not in
// the reference tree.
#pragma once

#define VPIPE_PLUGIN_ABI 8
#define VPIPE_PLUGIN_INFO_SCHEMA 1

// Host features a plugin may require beyond the ABI integer (README.md:
// "kernel-contract/1" and "accel-bag/1").
#define VPIPE_FEATURE_KERNEL_CONTRACT "kernel-contract/1"
#define VPIPE_FEATURE_ACCEL_BAG "accel-bag/1"

extern "C" {

// The plugin's identity, as the reference fills it (src/ltx25-plugin.cc:
// 59-68): schema, name, version, vendor, licence, summary, and the
// null-terminated list of required host features.
struct VpipePluginInfo {
  int schema;
  const char* name;
  const char* version;
  const char* vendor;
  const char* license;
  const char* summary;
  const char* const* requires_features;
};

}  // extern "C"

namespace vpipe {
class VpipePluginContext;
}

#define VPIPE_PLUGIN_EXPORT extern "C" __attribute__((visibility("default")))

// Defines the three symbols a host resolves: the ABI the plugin was built
// for, its info record, and the registration entry the host calls once with
// its context.
#define VPIPE_PLUGIN_DEFINE(info_ptr, register_fn)                                   \
  VPIPE_PLUGIN_EXPORT int vpipe_plugin_abi(void) { return VPIPE_PLUGIN_ABI; }         \
  VPIPE_PLUGIN_EXPORT const VpipePluginInfo* vpipe_plugin_info(void) { return (info_ptr); } \
  VPIPE_PLUGIN_EXPORT void vpipe_plugin_register(vpipe::VpipePluginContext* c) { register_fn(c); }
