/* HRM retrieval C ABI.  Same entry points and JSON as the reference integration ABI
 * (hrm_core/include/hrm/api.h:20-43 there) so existing ctypes / C callers work unchanged.
 *
 *  hrm_open(dir)        open a model directory holding router_index.bin + index.sqlite; NULL on failure
 *  hrm_query_json(...)  heap JSON string {prompt, cids, chosen[{sid,cid,rel,txt,txt_c}]}; free with hrm_free
 *  hrm_last_error()     message of the last failure on the calling thread (thread-local here)
 *
 * Handles are independent; one handle may be queried from several threads (queries are read-only). */
#pragma once
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct hrm_handle_t hrm_handle_t;

hrm_handle_t* hrm_open(const char* model_dir);
void hrm_close(hrm_handle_t* h);
char* hrm_query_json(hrm_handle_t* h, const char* prompt_utf8, int top_k, int top_m, int k, int lam_num,
                     int lam_den);
void hrm_free(void* p);
const char* hrm_last_error(void);

#ifdef __cplusplus
}
#endif
