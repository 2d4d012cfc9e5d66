/*
 * named_library.c -- body of every reference-named library file.
 *
 * The vLLM plugin loads libraries by the reference's file names
 * (src/gdn_state_codec/runtime.py:55-237).  Each such file built from this
 * source carries no code of its own: it is linked with a DT_NEEDED entry on
 * libgdn_state_codec_b200.so (found through RPATH $ORIGIN), so a dlsym() on
 * its handle resolves every statecentric_gdn_state_codec_* entry point from
 * the one CUDA library that implements them.
 */
const char statecentric_gdn_state_codec_backend_b200[] = "gdn-state-codec-b200 sm_100a";
