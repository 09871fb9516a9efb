;;;; cuda.lisp -- SBCL bindings of libembedcuda.so (sb-alien only, no new
;;;; dependencies).  Loaded after st/model/ann/kb, it lets the existing Lisp
;;;; entry points run on B200s:
;;;;
;;;;   (cuda:init)                        ; once, before model:load-model
;;;;   (cuda:load-model path)             ; instead of the weight reading of
;;;;                                      ; bert:load-model / llama:load-model
;;;;   (cuda:embed-ids ids)               ; one sequence of token ids
;;;;   (cuda:embed-batch list-of-id-vectors)
;;;;   (cuda:load-tokenizer "tokenizer.json") (cuda:embed-texts list-of-strings)
;;;;   (cuda:kmeans vecs sample k iters)  ; ann::kmeans
;;;;   (cuda:assign-all vecs n centroids k)
;;;;   (cuda:ann-build vecs sample k iters) ; kmeans + assign-all, rows sent once
;;;;   (cuda:index-load vecs n centroids counts lists)
;;;;   (cuda:index-load-files "index.bin" :ann-path "ann.bin" :dim 384)
;;;;   (cuda:ann-build-file "index.bin" "ann.bin" sample k iters)  ; ann:run
;;;;   (cuda:top-k q k)                   ; kb::top-k
;;;;   (cuda:kb-search "query" 8)         ; kb:kb-search, index resident on the GPU
;;;;
;;;; Every foreign call returns an int status; a negative status becomes a
;;;; Lisp ERROR carrying ec_last_error(), as st.lisp / model.lisp signal
;;;; theirs.  Arrays cross the boundary pinned (sb-sys:with-pinned-objects +
;;;; vector-sap); the library copies what it needs before returning.

(defpackage :cuda
  (:use :cl)
  (:export #:init #:available-p #:load-model #:dim #:embed-ids #:embed-batch
           #:load-tokenizer #:embed-texts
           #:kmeans #:assign-all #:ann-build #:index-load #:index-load-files #:ann-build-file
           #:top-k #:top-k-brute #:top-k-batch #:*nprobe*
           #:attach-kb #:kb-search))
(in-package :cuda)

(defparameter *library* (or (sb-ext:posix-getenv "EC_LIBRARY") "libembedcuda.so"))
(defparameter *nprobe* 64)   ; kb::*ann-nprobe*
(defvar *loaded* nil)
(defvar *dim* 0)
(defvar *ivf* nil)
(defvar *index-dim* 0)   ; dimension of the resident index (0: none loaded)

(defun available-p () *loaded*)

;;; ---- raw routines (include/embedcuda.h) ----------------------------------

(sb-alien:define-alien-routine ("ec_last_error" %last-error) sb-alien:c-string)
(sb-alien:define-alien-routine ("ec_init" %init) sb-alien:int
  (devices sb-sys:system-area-pointer) (ndev sb-alien:int))
(sb-alien:define-alien-routine ("ec_upload_tensor" %upload-tensor) sb-alien:int
  (name sb-alien:c-string) (dtype sb-alien:int) (shape sb-sys:system-area-pointer)
  (ndim sb-alien:int) (data sb-sys:system-area-pointer) (nbytes sb-alien:unsigned-long))
(sb-alien:define-alien-routine ("ec_load_model" %load-model) sb-alien:int
  (config sb-alien:c-string) (pooling sb-alien:c-string)
  (family sb-sys:system-area-pointer) (dim sb-sys:system-area-pointer))
(sb-alien:define-alien-routine ("ec_embed_batch" %embed-batch) sb-alien:int
  (ids sb-sys:system-area-pointer) (offsets sb-sys:system-area-pointer) (nseq sb-alien:int)
  (out sb-sys:system-area-pointer) (out-stride sb-alien:int))
(sb-alien:define-alien-routine ("ec_kmeans" %kmeans) sb-alien:int
  (x sb-sys:system-area-pointer) (n (sb-alien:signed 64)) (d sb-alien:int)
  (sample sb-sys:system-area-pointer) (nsample (sb-alien:signed 64)) (k sb-alien:int)
  (iters sb-alien:int) (init sb-sys:system-area-pointer) (centroids sb-sys:system-area-pointer))
(sb-alien:define-alien-routine ("ec_assign_all" %assign-all) sb-alien:int
  (x sb-sys:system-area-pointer) (n (sb-alien:signed 64)) (d sb-alien:int)
  (centroids sb-sys:system-area-pointer) (k sb-alien:int)
  (counts sb-sys:system-area-pointer) (lists sb-sys:system-area-pointer))
(sb-alien:define-alien-routine ("ec_ann_build" %ann-build) sb-alien:int
  (x sb-sys:system-area-pointer) (n (sb-alien:signed 64)) (d sb-alien:int)
  (sample sb-sys:system-area-pointer) (nsample (sb-alien:signed 64)) (k sb-alien:int)
  (iters sb-alien:int) (init sb-sys:system-area-pointer) (centroids sb-sys:system-area-pointer)
  (counts sb-sys:system-area-pointer) (lists sb-sys:system-area-pointer))
(sb-alien:define-alien-routine ("ec_index_load" %index-load) sb-alien:int
  (x sb-sys:system-area-pointer) (n (sb-alien:signed 64)) (d sb-alien:int)
  (centroids sb-sys:system-area-pointer) (k sb-alien:int)
  (counts sb-sys:system-area-pointer) (lists sb-sys:system-area-pointer))
(sb-alien:define-alien-routine ("ec_ivf_search" %ivf-search) sb-alien:int
  (q sb-sys:system-area-pointer) (nq sb-alien:int) (nprobe sb-alien:int) (topk sb-alien:int)
  (ids sb-sys:system-area-pointer) (scores sb-sys:system-area-pointer))
(sb-alien:define-alien-routine ("ec_flat_search" %flat-search) sb-alien:int
  (q sb-sys:system-area-pointer) (nq sb-alien:int) (topk sb-alien:int)
  (ids sb-sys:system-area-pointer) (scores sb-sys:system-area-pointer))

(sb-alien:define-alien-routine ("ec_index_load_files" %index-load-files) sb-alien:int
  (index-path sb-alien:c-string) (d sb-alien:int) (ann-path sb-alien:c-string)
  (n sb-sys:system-area-pointer))
(sb-alien:define-alien-routine ("ec_ann_build_file" %ann-build-file) sb-alien:int
  (index-path sb-alien:c-string) (d sb-alien:int) (k sb-alien:int) (iters sb-alien:int)
  (sample sb-sys:system-area-pointer) (nsample (sb-alien:signed 64))
  (ann-path sb-alien:c-string))

(sb-alien:define-alien-routine ("ec_tokenizer_from_json" %tokenizer-from-json) sb-alien:int
  (path sb-alien:c-string) (handle sb-sys:system-area-pointer))
(sb-alien:define-alien-routine ("ec_tokenize" %tokenize) sb-alien:int
  (handle sb-alien:int) (texts sb-sys:system-area-pointer) (lengths sb-sys:system-area-pointer)
  (ntexts sb-alien:int) (ids sb-sys:system-area-pointer) (cap (sb-alien:signed 64))
  (offsets sb-sys:system-area-pointer) (nthreads sb-alien:int))

(defun check (rc what)
  (when (minusp rc)
    (error "~A failed (status ~D): ~A" what rc (%last-error)))
  rc)

(defmacro with-saps (bindings &body body)
  "Bind each VAR to the SAP of a pinned specialised vector (or a null SAP)."
  `(sb-sys:with-pinned-objects ,(remove nil (mapcar #'second bindings))
     (let ,(mapcar (lambda (b)
                     `(,(first b) (if ,(second b)
                                      (sb-sys:vector-sap ,(second b))
                                      (sb-sys:int-sap 0))))
                   bindings)
       ,@body)))

;;; ---- context ---------------------------------------------------------------

(defun init (&optional devices)
  "Load the library and bring up DEVICES (list of CUDA ordinals; NIL = all)."
  (unless *loaded*
    (sb-alien:load-shared-object *library*)
    (let ((dv (and devices (coerce devices '(simple-array (signed-byte 32) (*))))))
      (with-saps ((p dv))
        (check (%init p (if dv (length dv) 0)) "ec_init")))
    (setf *loaded* t))
  t)

;;; ---- st.lisp: raw tensors straight to the device ---------------------------

(defun dtype-code (s)
  (cond ((string= s "F32") 0) ((string= s "BF16") 1) ((string= s "F16") 2)
        (t (error "unsupported dtype ~A" s))))

(defun upload-safetensors (path)
  "Hand every tensor's raw bytes to ec_upload_tensor (st:get-tensor without
the host widening, st.lisp:32-86)."
  (multiple-value-bind (header data-start) (st:parse-header path)
    (with-open-file (in path :direction :input :element-type '(unsigned-byte 8))
      (loop for name in (st:tensor-names header)
            for info = (gethash name header)
            unless (string= name "__metadata__")
              do (let* ((offs (gethash "data_offsets" info))
                        (nbytes (- (second offs) (first offs)))
                        (buf (make-array nbytes :element-type '(unsigned-byte 8)))
                        (shape (coerce (gethash "shape" info)
                                       '(simple-array (signed-byte 64) (*)))))
                   (file-position in (+ data-start (first offs)))
                   (unless (= (read-sequence buf in) nbytes)
                     (error "EOF in tensor ~A" name))
                   (with-saps ((sp shape) (bp buf))
                     (check (%upload-tensor name (dtype-code (gethash "dtype" info)) sp
                                            (length shape) bp nbytes)
                            (format nil "upload ~A" name))))))))

;;; ---- model.lisp ------------------------------------------------------------

(defun slurp (path)
  (when (probe-file path)
    (with-open-file (in path :direction :input :external-format :utf-8)
      (let ((s (make-string (file-length in))))
        (subseq s 0 (read-sequence s in))))))

(defun load-model (path)
  "Upload model.safetensors and build the model on the devices.  Returns the
family keyword as model:load-model does (model.lisp:28-46)."
  (init)
  (let* ((dir (make-pathname :defaults path :name nil :type nil))
         (cfg (slurp (merge-pathnames "config.json" dir)))
         (pool (slurp (merge-pathnames "1_Pooling/config.json" dir)))
         (fam (make-array 1 :element-type '(signed-byte 32)))
         (dm (make-array 1 :element-type '(signed-byte 32))))
    (upload-safetensors (merge-pathnames "model.safetensors" dir))
    (with-saps ((fp fam) (dp dm))
      (check (%load-model cfg pool fp dp) "ec_load_model"))
    (setf *dim* (aref dm 0))
    (ecase (aref fam 0) (1 :bert) (2 :mpnet) (3 :llama) (4 :gemma))))

(defun dim () *dim*)

(defun embed-batch (id-vectors)
  "List of token-id vectors -> list of L2-normalised (simple-array
single-float (dim)), in input order (model:embed for a whole batch)."
  (let* ((n (length id-vectors))
         (offsets (make-array (1+ n) :element-type '(signed-byte 64)))
         (total (reduce #'+ id-vectors :key #'length))
         (ids (make-array total :element-type '(signed-byte 32)))
         (out (make-array (* n *dim*) :element-type 'single-float)))
    (loop for v in id-vectors
          for i from 0
          with pos = 0
          do (setf (aref offsets i) pos)
             (loop for x across v do (setf (aref ids pos) x) (incf pos))
          finally (setf (aref offsets n) pos))
    (with-saps ((ip ids) (op offsets) (outp out))
      (check (%embed-batch ip op n outp *dim*) "ec_embed_batch"))
    (loop for i below n
          collect (subseq out (* i *dim*) (* (1+ i) *dim*)))))

(defun embed-ids (ids)
  "One sequence of token ids (tokenizer:tk-encode's output) -> embedding."
  (first (embed-batch (list ids))))

;;; ---- ann.lisp ----------------------------------------------------------------

(defun kmeans (vecs sample k iters &key (dim 384))
  "ann::kmeans (ann.lisp:79-125) on the GPUs.  SAMPLE is the vector of
training row indices; its first K rows initialise the centroids."
  (let* ((n (floor (length vecs) dim))
         (s (coerce sample '(simple-array (signed-byte 64) (*))))
         (cent (make-array (* k dim) :element-type 'single-float)))
    (with-saps ((xp vecs) (sp s) (cp cent) (np nil))
      (check (%kmeans xp n dim sp (length s) k iters np cp) "ec_kmeans"))
    cent))

(defun assign-all (vecs n centroids k &key (dim 384))
  "ann::assign-all (ann.lisp:127-158): (values counts lists)."
  (let ((counts (make-array k :element-type '(unsigned-byte 32)))
        (lists (make-array n :element-type '(unsigned-byte 32))))
    (with-saps ((xp vecs) (cp centroids) (np counts) (lp lists))
      (check (%assign-all xp n dim cp k np lp) "ec_assign_all"))
    (values counts lists)))

(defun ann-build (vecs sample k iters &key (dim 384))
  "The kmeans + assign-all pair of ann:run (ann.lisp:193-197) in one call:
(values centroids counts lists), the rows sent to the GPU once."
  (let* ((n (floor (length vecs) dim))
         (s (coerce sample '(simple-array (signed-byte 64) (*))))
         (cent (make-array (* k dim) :element-type 'single-float))
         (counts (make-array k :element-type '(unsigned-byte 32)))
         (lists (make-array n :element-type '(unsigned-byte 32))))
    (with-saps ((xp vecs) (sp s) (cp cent) (np nil) (kp counts) (lp lists))
      (check (%ann-build xp n dim sp (length s) k iters np cp kp lp) "ec_ann_build"))
    (values cent counts lists)))

;;; ---- kb.lisp -------------------------------------------------------------------

(defun index-load (vecs n &key centroids counts lists (dim 384))
  "Keep index.bin (and ann.bin when CENTROIDS is given) resident on the GPUs."
  (let ((k (if centroids (floor (length centroids) dim) 0)))
    (with-saps ((xp vecs) (cp centroids) (np counts) (lp lists))
      (check (%index-load xp n dim cp k np lp) "ec_index_load"))
    (setf *index-dim* dim
          *ivf* (plusp k))))

(defun index-load-files (index-path &key ann-path (dim 384))
  "kb::load-index's vectors + kb::load-ann straight from index.bin / ann.bin
into device memory (no Lisp array of the vectors).  Returns n."
  (let ((n (make-array 1 :element-type '(signed-byte 64))))
    (with-saps ((np n))
      (check (%index-load-files (namestring index-path) dim
                                (and ann-path (namestring ann-path)) np)
             "ec_index_load_files"))
    (setf *index-dim* dim
          *ivf* (and ann-path t))
    (aref n 0)))

(defun ann-build-file (index-path ann-path sample k iters &key (dim 384))
  "ann:run from index.bin to ann.bin in the library; SAMPLE is the vector of
training row ids (ann::random-sample's result), its first K rows the initial
centroids."
  (let ((sv (coerce sample '(simple-array (signed-byte 64) (*)))))
    (with-saps ((sp sv))
      (check (%ann-build-file (namestring index-path) dim k iters sp (length sv)
                              (namestring ann-path))
             "ec_ann_build_file"))))

(defvar *tokenizer* 0)
(defvar *have-tokenizer* nil)

(defun load-tokenizer (path)
  "make-tokenizer-from-json in the library; later EMBED-TEXTS calls use it."
  (let ((h (make-array 1 :element-type '(signed-byte 32))))
    (with-saps ((hp h))
      (check (%tokenizer-from-json (namestring path) hp) "ec_tokenizer_from_json"))
    (setf *have-tokenizer* t)
    (setf *tokenizer* (aref h 0))))

(defun embed-texts (texts)
  "tk-encode of every text on the library's host threads, then one batched
forward (model:embed for a list of texts, in input order)."
  (let* ((n (length texts))
         (octets (mapcar (lambda (s) (sb-ext:string-to-octets s :external-format :utf-8)) texts))
         (total (reduce #'+ octets :key #'length))
         (buf (make-array (max 1 total) :element-type '(unsigned-byte 8)))
         (lens (make-array n :element-type '(signed-byte 64)))
         (ptrs (make-array n :element-type '(unsigned-byte 64)))
         (offs (make-array (1+ n) :element-type '(signed-byte 64)))
         (ids (make-array (* 512 (max 1 n)) :element-type '(signed-byte 32))))
    (let ((pos 0) (i 0))
      (dolist (o octets)
        (replace buf o :start1 pos)
        (setf (aref lens i) (length o))
        (incf pos (length o))
        (incf i)))
    (sb-sys:with-pinned-objects (buf lens ptrs offs ids)
      (let ((base (sb-sys:sap-int (sb-sys:vector-sap buf))) (pos 0))
        (dotimes (i n)
          (setf (aref ptrs i) (+ base pos))
          (incf pos (aref lens i))))
      (check (%tokenize *tokenizer* (sb-sys:vector-sap ptrs) (sb-sys:vector-sap lens) n
                        (sb-sys:vector-sap ids) (length ids) (sb-sys:vector-sap offs) 0)
             "ec_tokenize"))
    (embed-batch (loop for i below n
                       collect (subseq ids (aref offs i) (aref offs (1+ i)))))))

(defun check-query (q)
  "The library reads *INDEX-DIM* floats per query and cannot see Q's length."
  (unless (= (length q) *index-dim*)
    (error "query of length ~D, the resident index has dim ~D" (length q) *index-dim*)))

(defun %search (q k ivf)
  (check-query q)
  (let ((ids (make-array k :element-type '(signed-byte 64)))
        (sc (make-array k :element-type 'single-float))
        (qv (coerce q '(simple-array single-float (*)))))
    (with-saps ((qp qv) (ip ids) (sp sc))
      (check (if ivf
                 (%ivf-search qp 1 *nprobe* k ip sp)
                 (%flat-search qp 1 k ip sp))
             "search"))
    (loop for i below k
          when (>= (aref ids i) 0)
            collect (cons (aref ids i) (aref sc i)))))

(defun top-k-brute (q k) (%search q k nil))

(defun top-k (q k)
  "kb::top-k (kb.lisp:366-368): list of (row . score), descending."
  (%search q k *ivf*))

(defun top-k-batch (queries k)
  "kb::top-k for a list of query vectors in one call (the library regroups a
large batch by probed list): a list with one (row . score) list per query,
each as top-k would return it."
  (mapc #'check-query queries)
  (let* ((nq (length queries))
         (d *index-dim*)
         (qv (make-array (* nq d) :element-type 'single-float))
         (ids (make-array (* nq k) :element-type '(signed-byte 64)))
         (sc (make-array (* nq k) :element-type 'single-float)))
    (loop for q in queries
          for i from 0
          do (replace qv (coerce q '(simple-array single-float (*))) :start1 (* i d)))
    (when (plusp nq)
      (with-saps ((qp qv) (ip ids) (sp sc))
        (check (if *ivf*
                   (%ivf-search qp nq *nprobe* k ip sp)
                   (%flat-search qp nq k ip sp))
               "search")))
    (loop for i below nq
          collect (loop for j from (* i k) below (* (1+ i) k)
                        when (>= (aref ids j) 0)
                          collect (cons (aref ids j) (aref sc j))))))

;;; ---- kb.lisp: kb-search with the index resident on the GPUs ---------------

(defvar *kb-attached* nil)

(defun attach-kb ()
  "Load kb's index as kb::load-index does (meta.tsv, texts.tsv offsets,
index.bin, ann.bin when present) and keep its vectors, centroids and lists
resident on the GPUs; afterwards TOP-K answers kb::top-k's queries there.
The model (CUDA:LOAD-MODEL or the patched model:load-model) is loaded here
when no model is, replacing kb::start-encoder (whose *encoder* flag
kb.lisp:205 reads but never binds)."
  (unless kb::*vectors* (kb::load-index))
  (when (zerop *dim*) (load-model (cfg:model-path)))
  (let ((d kb::*dim*))
    (if kb::*ann-centroids*
        (index-load kb::*vectors* kb::*n* :dim d
                    :centroids kb::*ann-centroids*
                    :counts (coerce kb::*ann-counts* '(simple-array (unsigned-byte 32) (*)))
                    :lists kb::*ann-lists*)
        (index-load kb::*vectors* kb::*n* :dim d)))
  (setf *nprobe* kb::*ann-nprobe*
        *kb-attached* t))

(defun kb-search (query &optional (k 8))
  "kb:kb-search (kb.lisp:202-211) on the GPUs: the query is embedded by the
library (its tokenizer when LOAD-TOKENIZER was called, else model:embed's
token ids) and searched over the resident index; returns the same plists
(:source :domain :score :text), best first."
  (unless *kb-attached* (attach-kb))
  (let ((q (if *have-tokenizer* (first (embed-texts (list query))) (model:embed query))))
    (loop for (idx . score) in (top-k q k)
          collect (list :source (aref kb::*sources* idx)
                        :domain (aref kb::*domains* idx)
                        :score score
                        :text (kb::chunk-text idx)))))
