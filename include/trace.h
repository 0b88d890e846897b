#ifndef PITORCH_TRACE_H
#define PITORCH_TRACE_H

/*
 * Host-side span tracing -- drop-in for pitorch/profiler/trace.h (same
 * struct layout and API). Spans wrap host calls (graph launches and their
 * synchronisation); per-kernel device timing comes from ncu. Chrome-trace
 * JSON output as in pitorch/profiler/trace.c:89-120.
 */

#include <stdint.h>

#define PT_TRACE_MAX_EVENTS  4096
#define PT_TRACE_MAX_DEPTH   32

typedef struct {
    const char *name;
    const char *cat;
    uint32_t    ts_us;
    uint32_t    dur_us;
    int8_t      layer;
    int8_t      depth;
    uint32_t    hw_cycles;
    uint32_t    hw_stall;
} pt_trace_event_t;

typedef struct {
    pt_trace_event_t events[PT_TRACE_MAX_EVENTS];
    int              count;
    int              enabled;
    struct {
        const char *name;
        const char *cat;
        uint32_t    ts_us;
        int8_t      layer;
    } stack[PT_TRACE_MAX_DEPTH];
    int              depth;
} pt_trace_t;

void pt_trace_init(pt_trace_t *t);
void pt_trace_begin(pt_trace_t *t, const char *name, const char *cat, int layer);
void pt_trace_end(pt_trace_t *t);
void pt_trace_reset(pt_trace_t *t);
uint32_t pt_time_us(void);
void pt_trace_write_json(const pt_trace_t *t, const char *path);
void pt_trace_write_meta(const char *path, const char *name,
                         const char *model, int dim, int layers,
                         int vocab, const char *device, int num_qpus,
                         int steps, float lr, float final_loss,
                         float total_time_s, const char *notes);

#endif
