/* The C ABI used from plain C (no Python, no PyTorch): configuration defaults, status strings, argument
 * validation without a device, and an engine brought up and shut down when a device is present.
 * Built and run by tests/test_c_abi.py:  cc -I include tests/c_abi/abi_smoke.c -L<lib dir> -lud */
#include <stdio.h>
#include <string.h>

#include "ud.h"

int main(void) {
    ud_config cfg;
    ud_config_default(&cfg);
    if (cfg.n_layers != 24 || cfg.d_model != 1024 || cfg.joint_dim != 640 || cfg.vocab != 1025) {
        printf("bad defaults\n");
        return 1;
    }
    if (strcmp(ud_status_string(UD_OK), "ok") != 0) {
        printf("bad status string\n");
        return 1;
    }
    /* an invalid configuration is rejected before any device is touched */
    ud_config bad = cfg;
    bad.max_chunk_frames = 64;
    ud_engine* e = NULL;
    if (ud_init(&bad, 0, &e) != UD_ERR_INVALID_ARGUMENT || e != NULL) {
        printf("invalid config accepted\n");
        return 1;
    }
    /* NULL handles are statuses */
    if (ud_step_sync(NULL) != UD_ERR_INVALID_ARGUMENT || ud_synchronize(NULL) != UD_ERR_INVALID_ARGUMENT) {
        printf("NULL engine not rejected\n");
        return 1;
    }
    /* a small engine: on a machine without a device the status says so, on a B200 it comes up */
    cfg.n_layers = 0;
    cfg.sub_channels = 0;
    cfg.joint_dim = 0;
    cfg.max_streams = 2;
    cfg.max_batch = 2;
    ud_status s = ud_init(&cfg, 0, &e);
    if (s == UD_OK) {
        ud_stream_id id = -1;
        if (ud_stream_open(e, 1, &id) != UD_OK || id < 0) {
            printf("stream open failed\n");
            return 1;
        }
        ud_stream_close(e, id);
        ud_shutdown(e);
        printf("engine ok\n");
    } else {
        char msg[256];
        ud_last_error(msg, sizeof msg);
        printf("no engine: %s (%s)\n", ud_status_string(s), msg);
        if (s != UD_ERR_CUDA) return 1;
    }
    return 0;
}
